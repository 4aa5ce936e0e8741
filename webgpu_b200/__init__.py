"""webgpu_b200 — a B200-native (sm_100a) implementation of the ahpah-dev/WebGPU
runtime's per-token decoder loop, behind the same SDK surface.

    from webgpu_b200 import WebGPU
    rt = WebGPU()
    rt.load("model.gguf", {"contextLength": 4096, "batchSize": 128})
    for ev in rt.generate([{"role": "user", "content": "hi"}], {"temperature": 0}):
        print(ev.delta, end="")

The device work runs in libwgd.so (C ABI in include/wgd.h); this package is the
host half: GGUF reader, context policy, engine loop and SDK/worker protocol.
"""
from .engine import AbortError, ModelInfo, PagedEngine, TokenEvent, sample  # noqa: F401
from .sdk import WebGPU  # noqa: F401

__all__ = ["WebGPU", "PagedEngine", "TokenEvent", "ModelInfo", "AbortError", "sample"]
