"""PagedEngine: the host half of the decoder loop.

A mirror of the reference's PagedEngine (src/core/engine.ts:26-304,
ahpah-dev/WebGPU 0.9.0): the same presets, option validation, prefix reuse,
prompt-batch prefill, streamed greedy/temperature generation and error
messages. The device half — WebGPU buffers, WGSL dispatches and weight-page
uploads — is replaced by the CUDA library (include/wgd.h), called once per
forward.

Deliberate differences, for a B200 host: the GPU budget ceiling is the device's
memory (the reference caps it at a browser's 16 GiB); `LoadOptions` adds
`tensorParallel`/`rank`/`device`/`exchange` for multi-GPU runs; `generate_ids`
drives token ids directly, which the benchmark configurations (no tokenizer metadata) use.
"""
from __future__ import annotations

import ctypes
import math
import random
import time
from dataclasses import dataclass, field

import numpy as np

from . import _native
from .context import MAX_CONTEXT, MAX_MESSAGE_CHARS, attention_memory, output_limit, suggest_budget, validate_context
from .gguf import model_config, read_gguf, to_native_config
from .source import make_source
from .tokenizer import make_tokenizer

MiB = 1024 ** 2
# engine.ts:14-18
PRESETS = {"lite": {"budget": 512, "batch": 8, "page": 16},
           "low-memory": {"budget": 2048, "batch": 16, "page": 16},
           "fast": {"budget": 6144, "batch": 128, "page": 64}}
MAX_BUDGET_MIB = 180 * 1024  # one B200's HBM; the browser reference stops at 16384


def _is_number(v) -> bool:
    """A JavaScript number: int or float, but not bool (Number.isFinite(true) is false)."""
    return isinstance(v, (int, float)) and not isinstance(v, bool)


def _is_integer(v) -> bool:
    """Number.isInteger: an integral number (2.0 counts), never a bool or a string."""
    return _is_number(v) and math.isfinite(v) and float(v).is_integer()


class AbortError(Exception):
    """Raised when a request is cancelled (the reference's AbortError, sdk.ts:27)."""


@dataclass
class TokenEvent:
    """engine.ts:24"""
    token: int
    text: str
    delta: str
    tokens: int
    promptTokens: int
    contextLength: int
    seconds: float
    stats: dict


@dataclass
class ModelInfo:
    """engine.ts:23"""
    config: object
    fileBytes: int
    adapter: str
    contextLength: int
    gpuBudgetMiB: int
    batchSize: int
    performance: str
    stats: dict
    tensorParallel: int = 1


def sample(logits, temperature: float, top_k: int, top_p: float, rng=random.random) -> int:
    """engine.ts:305-324 for a host row of logits, drawn on the device (wgd_op_sample) with one
    uniform number from `rng` (Math.random()). Raises the reference's error when no logit is
    finite. The engine itself never reads logits back: generate draws with wgd_forward_sample."""
    import torch

    x = torch.as_tensor(np.ascontiguousarray(logits, dtype=np.float32)).cuda()
    tok = ctypes.c_int32(-1)
    st = _native.lib().wgd_op_sample(x.data_ptr(), x.numel(), float(temperature), int(top_k), float(top_p), rng(),
                                     ctypes.byref(tok), None)
    if st == _native.WGD_ENONFINITE:
        raise ValueError(_native.last_error())
    _native.check(st, "sample")
    return tok.value


class PagedEngine:
    def __init__(self, progress=None):
        self.progress = progress or (lambda p: None)
        self.ctx = None
        self.source = None
        self.gguf = None
        self.config = None
        self.tokenizer = None
        self.context = 512
        self.batch = 16
        self.budget = 2048
        self.performance = "low-memory"
        self.busy = False
        self.disposed = False
        self.tokens_in_cache: list[int] = []
        self.kv_capacities: list[int] = []
        self.tp = 1
        self.rank = 0
        self.device = 0
        self._logits = None
        self.random = random.random  # the uniform draw per sampled token (Math.random())

    # ------------------------------------------------------------------ load
    def load(self, src, options: dict | None = None, signal=None) -> ModelInfo:
        """engine.ts:51-114."""
        o = dict(options or {})
        self.performance = o.get("performance", "low-memory")
        if self.performance not in PRESETS:
            raise ValueError("Performance must be lite, low-memory or fast.")
        preset = PRESETS[self.performance]
        self.context = o.get("contextLength", 512)
        self.batch = o.get("batchSize", preset["batch"])
        validate_context(self.context)
        if self.batch not in (1, 8, 16, 32, 64, 128):
            raise ValueError("Batch size must be 1, 8, 16, 32, 64 or 128.")
        b = o.get("gpuBudgetMiB")
        if b is not None and (not isinstance(b, int) or b < 512 or b > MAX_BUDGET_MIB):
            raise ValueError(f"GPU budget must be 512–{MAX_BUDGET_MIB} MiB.")
        self.tp = int(o.get("tensorParallel", 1))
        self.rank = int(o.get("rank", 0))
        self.device = int(o.get("device", self.rank))
        self.source = make_source(src)
        self.progress({"phase": "loading", "detail": "Reading GGUF metadata and tokenizer", "fraction": 0.05})
        self.gguf = read_gguf(self.source)
        self.config = c = model_config(self.gguf)
        validate_context(self.context, c.max_context)
        self.budget = b if b is not None else suggest_budget(self.source.size, self.performance)
        if not isinstance(self.budget, int) or self.budget < 512 or self.budget > MAX_BUDGET_MIB:
            raise ValueError(f"GPU budget must be 512–{MAX_BUDGET_MIB} MiB.")
        self.tokenizer = make_tokenizer(self.gguf.metadata, c.family)
        memory = attention_memory(c, self.context, self.batch)
        self.kv_capacities = memory["capacities"]
        kv_per_rank = memory["total_bytes"] // self.tp
        if kv_per_rank + 256 * MiB > self.budget * MiB:
            raise ValueError(f"A {self.context:,}-token context needs {math.ceil(kv_per_rank / MiB):,} MiB of attention state "
                             f"plus working memory. Choose at least {math.ceil((kv_per_rank + 256 * MiB) / MiB):,} MiB of GPU "
                             f"budget, or reduce context.")
        L = _native.lib()
        status = ctypes.c_int(0)
        self.ctx = L.wgd_create(self.device, self.rank, self.tp, self.budget * MiB, preset["page"] * MiB, ctypes.byref(status))
        if not self.ctx:
            _native.check(status.value, "wgd_create")
        try:
            self.progress({"phase": "loading", "detail": "Placing weights on the GPU", "fraction": 0.25})
            cfg = to_native_config(c)
            _native.check(L.wgd_model_begin(self.ctx, ctypes.byref(cfg), self.context, self.batch), "model_begin")
            for t in self.gguf.tensors.values():
                dims = (ctypes.c_uint64 * 4)(*t.dims, *([0] * (4 - len(t.dims))))
                _native.check(L.wgd_tensor_register(self.ctx, t.name.encode(), t.type, dims, len(t.dims), t.offset, t.bytes,
                                                    t.row_bytes), "tensor_register")
            _native.check(L.wgd_model_end(self.ctx), "model_end")
            if self.tp > 1:
                self._open_peers(o.get("exchange"))
            if o.get("pull"):
                self._pull()
            else:
                self._upload(signal)
            ready = ctypes.c_int(0)
            _native.check(L.wgd_model_ready(self.ctx, ctypes.byref(ready)), "model_ready")
            if not ready.value:
                raise RuntimeError("weights incomplete after load")
            self.progress({"phase": "ready", "detail": "Ready.", "fraction": 1.0, "stats": self.stats()})
            return self.info()
        except BaseException:
            self.dispose()
            raise

    def _open_peers(self, exchange):
        """Exchanges the device handles of the tensor-parallel exchange buffers.
        `exchange(bytes) -> list[bytes]` is an all-gather over the ranks."""
        if exchange is None:
            raise ValueError("tensorParallel > 1 needs an 'exchange' all-gather callable")
        L = _native.lib()
        n = L.wgd_tp_handle_size()
        buf = ctypes.create_string_buffer(n)
        _native.check(L.wgd_tp_export(self.ctx, buf), "tp_export")
        handles = exchange(bytes(buf.raw))
        if len(handles) != self.tp:
            raise RuntimeError("handle exchange returned the wrong number of ranks")
        allh = b"".join(handles)
        _native.check(L.wgd_tp_open_peers(self.ctx, ctypes.c_char_p(allh)), "tp_open_peers")

    def _pull(self):
        """Loads through the library's page reader: the library asks for byte ranges of the model
        (ByteSource.read, source.ts:2-6) in pages of whole rows."""
        L = _native.lib()
        src = self.source

        def read(_user, offset, length, dst):
            try:
                data = src.read(offset, length)
                ctypes.memmove(dst, bytes(data) if not isinstance(data, (bytes, bytearray)) else data, length)
                return 0
            except Exception:  # reported by the library as an I/O error
                return 1

        self._reader = _native.READ_FN(read)  # kept alive while the context exists
        _native.check(L.wgd_set_page_reader(self.ctx, self._reader, None), "set_page_reader")
        _native.check(L.wgd_load_weights(self.ctx), "load_weights")

    def _upload(self, signal=None):
        L = _native.lib()
        view = self.source.view()
        tensors = list(self.gguf.tensors.values())
        for i, t in enumerate(tensors):
            if signal is not None and signal.is_set():
                raise AbortError("Stopped by user")
            if view is not None:
                ptr = view.ctypes.data + t.offset
                if t.bytes <= 64 * MiB or len(t.dims) == 1:
                    _native.check(L.wgd_tensor_upload(self.ctx, t.name.encode(), 0, ctypes.c_void_p(ptr), t.bytes), "upload")
                else:
                    step = max(1, (64 * MiB) // t.row_bytes) * t.row_bytes
                    for off in range(0, t.bytes, step):
                        n = min(step, t.bytes - off)
                        _native.check(L.wgd_tensor_upload(self.ctx, t.name.encode(), off, ctypes.c_void_p(ptr + off), n), "upload")
            else:
                step = max(1, (64 * MiB) // t.row_bytes) * t.row_bytes if len(t.dims) > 1 else t.bytes
                for off in range(0, t.bytes, step):
                    n = min(step, t.bytes - off)
                    data = bytes(self.source.read(t.offset + off, n))
                    _native.check(L.wgd_tensor_upload(self.ctx, t.name.encode(), off, data, n), "upload")
            if i % 20 == 0:
                self.progress({"phase": "loading", "detail": "Uploading weights", "fraction": 0.3 + 0.65 * i / len(tensors)})

    def info(self) -> ModelInfo:
        return ModelInfo(self.config, self.source.size, "NVIDIA B200 (wgd)", self.context, self.budget, self.batch,
                         self.performance, self.stats(), self.tp)

    def stats(self) -> dict:
        """PagingStats (pager.ts:5) plus device timings."""
        if not self.ctx:
            return {}
        s = _native.StatsC()
        _native.check(_native.lib().wgd_stats_get(self.ctx, ctypes.byref(s)), "stats")
        return {"readBytes": s.read_bytes, "readMs": s.read_ms, "uploads": s.uploads, "cacheHits": s.cache_hits,
                "cacheBytes": s.cache_bytes, "gpuBytes": s.gpu_bytes, "peakGpuBytes": s.peak_gpu_bytes,
                "pageBytes": s.page_bytes, "forwards": s.forwards, "tokens": s.tokens, "lastForwardMs": s.last_forward_ms,
                "streamedBytes": s.streamed_bytes}

    # --------------------------------------------------------------- forward
    def forward(self, ids, start: int, logits: bool, want_logits: bool = False):
        """engine.ts:138-180 — one device call. Returns the greedy token id of the last
        row (and the logits when want_logits) or None when logits is False."""
        L = _native.lib()
        n = len(ids)
        arr = (ctypes.c_int32 * n)(*ids)
        out = ctypes.c_int32(-1)
        want = 0 if not logits else (2 if want_logits else 1)
        lp = None
        if want == 2:
            if self._logits is None:
                self._logits = np.zeros(self.config.vocab, dtype=np.float32)
            lp = self._logits.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        st = L.wgd_forward(self.ctx, arr, n, start, want, ctypes.byref(out), lp)
        if st == _native.WGD_ECANCELLED:
            raise AbortError("Stopped by user")
        if st == _native.WGD_ENONFINITE:
            raise ValueError(_native.last_error())
        _native.check(st, "forward")
        if want == 0:
            return None
        return (out.value, self._logits.copy()) if want == 2 else out.value

    def forward_sample(self, ids, start: int, temperature: float, top_k: int, top_p: float) -> int:
        """engine.ts:138-180 and sample() (engine.ts:305-324) in one device call: the token is
        drawn on the device from the last row's logits with one uniform number from
        self.random (Math.random()); only the token id comes back."""
        L = _native.lib()
        n = len(ids)
        arr = (ctypes.c_int32 * n)(*ids)
        out = ctypes.c_int32(-1)
        st = L.wgd_forward_sample(self.ctx, arr, n, start, float(temperature), int(top_k), float(top_p), self.random(),
                                  ctypes.byref(out))
        if st == _native.WGD_ECANCELLED:
            raise AbortError("Stopped by user")
        if st == _native.WGD_ENONFINITE:
            raise ValueError(_native.last_error())
        _native.check(st, "forward_sample")
        return out.value

    # --------------------------------------------------------------- generate
    def generate(self, messages, options: dict | None = None, signal=None):
        """engine.ts:257-301."""
        if self.busy:
            raise RuntimeError("A generation is already running.")
        if self.disposed or not self.ctx:
            raise RuntimeError("Load a model first.")
        if (not isinstance(messages, list) or not messages
                or any(m.get("role") not in ("user", "assistant") or not isinstance(m.get("content"), str)
                       or len(m["content"]) > MAX_MESSAGE_CHARS for m in messages)):
            raise ValueError(f"Provide user/assistant text messages (at most {MAX_MESSAGE_CHARS:,} characters each).")
        prompt = self.tokenizer.chat(messages)
        yield from self._generate(prompt, options or {}, signal)

    def generate_ids(self, prompt_ids, options: dict | None = None, signal=None):
        """Token-id entry point (no tokenizer): the same loop as generate."""
        if self.busy:
            raise RuntimeError("A generation is already running.")
        if self.disposed or not self.ctx:
            raise RuntimeError("Load a model first.")
        prompt = [int(i) for i in prompt_ids]
        if not prompt:
            raise ValueError("The prompt has no tokens.")
        yield from self._generate(prompt, options or {}, signal)

    def _generate(self, prompt, options, signal):
        max_tokens = options.get("maxTokens", 128)
        if not _is_integer(max_tokens) or max_tokens < 1 or max_tokens > MAX_CONTEXT:
            raise ValueError(f"maxTokens must be 1–{MAX_CONTEXT}.")
        temperature = options.get("temperature", 0.7)
        top_k = options.get("topK", 40)
        top_p = options.get("topP", 0.9)
        if (not _is_number(temperature) or not math.isfinite(temperature) or temperature < 0 or temperature > 2
                or not _is_integer(top_k) or top_k < 1 or top_k > 200
                or not _is_number(top_p) or not math.isfinite(top_p) or top_p <= 0 or top_p > 1):
            raise ValueError("Invalid sampling settings.")
        max_tokens, top_k = int(max_tokens), int(top_k)
        self.busy = True
        try:
            limit = output_limit(max_tokens, len(prompt), self.context)
            shared = 0
            while shared < len(prompt) and shared < len(self.tokens_in_cache) and prompt[shared] == self.tokens_in_cache[shared]:
                shared += 1
            shared = min(shared, len(prompt) - 1)
            if shared < len(self.tokens_in_cache) and any(cap < self.context for cap in self.kv_capacities):
                shared = 0
            started = time.perf_counter()
            self.tokens_in_cache = self.tokens_in_cache[:shared]
            greedy = temperature == 0
            result = None
            for i in range(shared, len(prompt), self.batch):
                if signal is not None and signal.is_set():
                    raise AbortError("Stopped by user")
                batch = prompt[i:i + self.batch]
                last = i + len(batch) == len(prompt)
                if last and not greedy:
                    result = self.forward_sample(batch, i, temperature, top_k, top_p)
                else:
                    result = self.forward(batch, i, last)
                self.tokens_in_cache += batch
            generated: list[int] = []
            text = ""
            for i in range(limit):
                if signal is not None and signal.is_set():
                    raise AbortError("Stopped by user")
                token = result
                if token in self.tokenizer.eos:
                    break
                generated.append(token)
                full = self.tokenizer.decode(generated) if self.tokenizer.usable else ""
                delta = full[len(text):]
                text = full
                yield TokenEvent(token, text, delta, len(generated), len(prompt), self.context,
                                 time.perf_counter() - started, self.stats())
                if i + 1 < limit:
                    pos = len(self.tokens_in_cache)
                    result = (self.forward([token], pos, True) if greedy else
                              self.forward_sample([token], pos, temperature, top_k, top_p))
                    self.tokens_in_cache.append(token)
        except BaseException:
            self.tokens_in_cache = []
            raise
        finally:
            self.busy = False

    def reset(self):
        """engine.ts:302"""
        if self.busy:
            raise RuntimeError("Stop generation first.")
        self.tokens_in_cache = []
        if self.ctx:
            _native.lib().wgd_truncate_kv(self.ctx, 0)

    def cancel(self):
        if self.ctx:
            _native.lib().wgd_cancel(self.ctx)

    def dispose(self):
        """engine.ts:303"""
        self.disposed = True
        if self.ctx:
            _native.lib().wgd_destroy(self.ctx)
            self.ctx = None
        self.tokens_in_cache = []
