"""Seeded synthetic GGUF models and weight blocks.

The benchmark configurations are random-init models of real architectures; no
checkpoint is downloaded. This module writes complete GGUF images (header,
metadata, tensor directory, aligned tensor data) whose weights come from the
seeded generator in ``quantize.c``:

* ``tiny_dense(kind)`` restates the three F32 check models of the reference's
  ``scripts/verify-dense.mjs:25,60-135`` (LCG seeds 7/11/13, byte alphabet
  vocabulary, chat-framed prompts), so the same prompts can be decoded here.
* ``baseline_spec(i)`` gives the architectures of the benchmark configurations
  (tiny llama F32, Qwen2.5-0.5B, Llama-3-8B, Gemma-3-27B shapes).

GGUF is written in the layout the reference parser reads
(``src/core/gguf.ts:85-114``): version 3, little-endian, 32-byte alignment.
"""
from __future__ import annotations

import ctypes
import math
import os
import struct
from dataclasses import dataclass, field

import numpy as np

from .._build_paths import synth_lib_path

F32, F16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 2, 8, 12, 13, 14
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}
TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}

_LIB = None


def lib():
    """The native generator; raises if the shared library has not been built."""
    global _LIB
    if _LIB is None:
        path = synth_lib_path()
        if not os.path.exists(path):
            raise RuntimeError(f"synthetic-weight library missing: {path} (run __graft_entry__.build())")
        L = ctypes.CDLL(path)
        i64, u64, vp = ctypes.c_int64, ctypes.c_uint64, ctypes.c_void_p
        L.synth_normal_quantized.restype = i64
        L.synth_normal_quantized.argtypes = [ctypes.c_int, i64, i64, u64, u64, ctypes.c_double, ctypes.c_double, vp]
        L.synth_quantize.restype = i64
        L.synth_quantize.argtypes = [ctypes.c_int, vp, i64, i64, vp]
        L.synth_random_blocks.restype = i64
        L.synth_random_blocks.argtypes = [ctypes.c_int, i64, u64, u64, ctypes.c_double, vp]
        L.synth_fill_normal.restype = None
        L.synth_fill_normal.argtypes = [vp, i64, u64, u64, ctypes.c_double, ctypes.c_double]
        L.synth_fill_ints.restype = None
        L.synth_fill_ints.argtypes = [vp, i64, u64, u64, ctypes.c_int32]
        L.synth_set_threads.restype = None
        L.synth_set_threads.argtypes = [ctypes.c_int]
        # every visible core, also under a launcher that exports OMP_NUM_THREADS=1 (the bytes do
        # not depend on the thread count)
        try:
            L.synth_set_threads(len(os.sched_getaffinity(0)))
        except AttributeError:
            L.synth_set_threads(os.cpu_count() or 1)
        _LIB = L
    return _LIB


def row_bytes(ggml_type: int, cols: int) -> int:
    be, bb = BLOCK[ggml_type]
    assert cols % be == 0, (ggml_type, cols)
    return cols // be * bb


def quantize(ggml_type: int, x: np.ndarray) -> np.ndarray:
    """Packs a float32 [rows, cols] array into GGUF block bytes (uint8 [rows, row_bytes])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    rows, cols = x.shape
    out = np.zeros((rows, row_bytes(ggml_type, cols)), dtype=np.uint8)
    n = lib().synth_quantize(ggml_type, x.ctypes.data, rows, cols, out.ctypes.data)
    if n < 0:
        raise ValueError("bad quantisation shape")
    return out


def normal_quantized(ggml_type: int, rows: int, cols: int, seed: int, stream: int, std: float = 0.02,
                     mean: float = 0.0, out: np.ndarray | None = None) -> np.ndarray:
    """N(mean, std) weights generated and packed block by block (row-major [rows][cols])."""
    nbytes = rows * row_bytes(ggml_type, cols)
    if out is None:
        out = np.empty(nbytes, dtype=np.uint8)
    assert out.nbytes >= nbytes and out.flags.c_contiguous
    n = lib().synth_normal_quantized(ggml_type, rows, cols, seed, stream, mean, std, out.ctypes.data)
    if n != nbytes:
        raise ValueError("bad quantisation shape")
    return out


def random_blocks(ggml_type: int, nblocks: int, seed: int, stream: int = 0, scale_std: float = 1e-3) -> np.ndarray:
    """GEMV microbench blocks with uniform fields and |N(0, scale_std)| fp16 scales."""
    out = np.empty(nblocks * BLOCK[ggml_type][1], dtype=np.uint8)
    lib().synth_random_blocks(ggml_type, nblocks, seed, stream, scale_std, out.ctypes.data)
    return out


def normal(n: int, seed: int, stream: int, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().synth_fill_normal(out.ctypes.data, n, seed, stream, mean, std)
    return out


def uniform_ids(n: int, vocab: int, seed: int, stream: int = 0xC0FFEE) -> list[int]:
    out = np.empty(n, dtype=np.int32)
    lib().synth_fill_ints(out.ctypes.data, n, seed, stream, vocab)
    return [int(v) for v in out]


# --------------------------------------------------------------------------- GGUF

GGUF_MAGIC = 0x46554747
T_U32, T_I32, T_F32V, T_BOOL, T_STR, T_ARR, T_U64 = 4, 5, 6, 7, 8, 9, 10


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v) -> bytes:
    if vtype == T_U32:
        return struct.pack("<I", v)
    if vtype == T_I32:
        return struct.pack("<i", v)
    if vtype == T_F32V:
        return struct.pack("<f", v)
    if vtype == T_BOOL:
        return struct.pack("<B", 1 if v else 0)
    if vtype == T_STR:
        return _str(v)
    if vtype == T_U64:
        return struct.pack("<Q", v)
    raise ValueError(vtype)


@dataclass
class TensorSpec:
    name: str
    dims: tuple          # GGUF order: (cols, rows) for matrices, (n,) for vectors
    ggml_type: int
    init: str = "normal"  # "normal" | "ones" | "lcg" | "raw"
    std: float = 0.02
    stream: int = 0
    data: np.ndarray | None = None  # float32 values ("lcg") or raw bytes ("raw")

    @property
    def n(self) -> int:
        return int(np.prod(self.dims))

    @property
    def nbytes(self) -> int:
        be, bb = BLOCK[self.ggml_type]
        return self.n // be * bb


@dataclass
class ModelSpec:
    architecture: str
    metadata: list            # [(key, vtype, value)] or [(key, T_ARR, (elem_type, values))]
    tensors: list[TensorSpec]
    seed: int = 0
    prompt: list[int] = field(default_factory=list)
    description: str = ""


def _metadata_bytes(metadata) -> bytes:
    out = bytearray()
    for key, vtype, value in metadata:
        out += _str(key) + struct.pack("<I", vtype)
        if vtype == T_ARR:
            etype, values = value
            out += struct.pack("<IQ", etype, len(values))
            for v in values:
                out += _value(etype, v)
        else:
            out += _value(vtype, value)
    return bytes(out)


def _align(n: int, a: int = 32) -> int:
    return (n + a - 1) // a * a


def build_gguf(spec: ModelSpec, threads_hint: int | None = None) -> np.ndarray:
    """Writes the full GGUF image into one uint8 array (header + aligned tensor data)."""
    infos = bytearray()
    offset = 0
    placed = []
    for t in spec.tensors:
        offset = _align(offset)
        placed.append((t, offset))
        infos += _str(t.name) + struct.pack("<I", len(t.dims))
        for d in t.dims:
            infos += struct.pack("<Q", d)
        infos += struct.pack("<IQ", t.ggml_type, offset)
        offset += t.nbytes
    head = struct.pack("<IIQQ", GGUF_MAGIC, 3, len(spec.tensors), len(spec.metadata)) + _metadata_bytes(spec.metadata) + bytes(infos)
    data_start = _align(len(head))
    image = np.zeros(data_start + _align(offset), dtype=np.uint8)
    image[: len(head)] = np.frombuffer(head, dtype=np.uint8)
    for t, off in placed:
        dst = image[data_start + off: data_start + off + t.nbytes]
        cols = t.dims[0]
        rows = t.n // cols
        if t.init == "raw":
            dst[:] = np.frombuffer(np.ascontiguousarray(t.data).tobytes(), dtype=np.uint8)
        elif t.init == "ones":
            dst[:] = quantize(t.ggml_type, np.ones((rows, cols), np.float32)).reshape(-1)
        elif t.init == "lcg":
            dst[:] = quantize(t.ggml_type, np.asarray(t.data, np.float32).reshape(rows, cols)).reshape(-1)
        else:
            normal_quantized(t.ggml_type, rows, cols, spec.seed, t.stream, t.std, out=dst)
    return image


def write_gguf(spec: ModelSpec, path: str) -> int:
    image = build_gguf(spec)
    with open(path, "wb") as f:
        f.write(image.tobytes())
    return image.nbytes


# ----------------------------------------------------------- architecture specs

def _arch_metadata(arch: str, *, layers, hidden, ffn, heads, kv_heads, head_dim, eps, theta, context=32768,
                   rope_dim=None, extra=()):
    md = [
        ("general.architecture", T_STR, arch),
        ("general.name", T_STR, f"synthetic-{arch}"),
        ("general.file_type", T_U32, 15),
        (f"{arch}.block_count", T_U32, layers),
        (f"{arch}.context_length", T_U32, context),
        (f"{arch}.embedding_length", T_U32, hidden),
        (f"{arch}.feed_forward_length", T_U32, ffn),
        (f"{arch}.attention.head_count", T_U32, heads),
        (f"{arch}.attention.head_count_kv", T_U32, kv_heads),
        (f"{arch}.attention.key_length", T_U32, head_dim),
        (f"{arch}.attention.layer_norm_rms_epsilon", T_F32V, eps),
        (f"{arch}.rope.dimension_count", T_U32, rope_dim or head_dim),
        (f"{arch}.rope.freq_base", T_F32V, theta),
    ]
    md.extend(extra)
    return md


def dense_spec(arch: str, *, seed: int, layers: int, hidden: int, ffn: int, heads: int, kv_heads: int, head_dim: int,
               vocab: int, eps: float, theta: float, wtype: int = F32, out_type: int | None = None,
               embd_type: int | None = None, bias: bool = False, qk_norm: bool = False, tied: bool = False,
               gate: bool = True, std: float = 0.02, context: int = 32768, type_for=None, extra=()) -> ModelSpec:
    """A llama/qwen2/qwen3-family model with N(0, std) matrices and unit norms.
    `type_for(name, cols)` may override the block type of one matrix."""
    q, kv = heads * head_dim, kv_heads * head_dim
    stream = [0]

    def mat(name, cols, rows, ggml_type):
        if type_for:
            ggml_type = type_for(name, cols, ggml_type)
        stream[0] += 1
        return TensorSpec(name, (cols, rows), ggml_type, "normal", std, stream[0])

    def vec(name, n, init="ones"):
        stream[0] += 1
        return TensorSpec(name, (n,), F32, init, std, stream[0])

    embd_type = wtype if embd_type is None else embd_type
    out_type = wtype if out_type is None else out_type
    tensors = [mat("token_embd.weight", hidden, vocab, embd_type), vec("output_norm.weight", hidden)]
    if not tied:
        tensors.append(mat("output.weight", hidden, vocab, out_type))
    for l in range(layers):
        p = f"blk.{l}."
        tensors += [vec(p + "attn_norm.weight", hidden), mat(p + "attn_q.weight", hidden, q, wtype),
                    mat(p + "attn_k.weight", hidden, kv, wtype), mat(p + "attn_v.weight", hidden, kv, wtype),
                    mat(p + "attn_output.weight", q, hidden, wtype)]
        if bias:
            tensors += [vec(p + "attn_q.bias", q, "normal"), vec(p + "attn_k.bias", kv, "normal"), vec(p + "attn_v.bias", kv, "normal")]
        if qk_norm:
            tensors += [vec(p + "attn_q_norm.weight", head_dim), vec(p + "attn_k_norm.weight", head_dim)]
        tensors.append(vec(p + "ffn_norm.weight", hidden))
        if gate:
            tensors.append(mat(p + "ffn_gate.weight", hidden, ffn, wtype))
        tensors += [mat(p + "ffn_up.weight", hidden, ffn, wtype), mat(p + "ffn_down.weight", ffn, hidden, wtype)]
    md = _arch_metadata(arch, layers=layers, hidden=hidden, ffn=ffn, heads=heads, kv_heads=kv_heads,
                        head_dim=head_dim, eps=eps, theta=theta, context=context, extra=extra)
    return ModelSpec(arch, md, tensors, seed=seed)


def gemma_spec(*, seed: int, layers: int, hidden: int, ffn: int, heads: int, kv_heads: int, head_dim: int, vocab: int,
               eps: float = 1e-6, theta: float = 1e6, local_theta: float = 1e4, window: int = 1024,
               wtype: int = Q4_K, embd_type: int = Q6_K, std: float = 0.02, context: int = 131072) -> ModelSpec:
    """A Gemma-3 model (tied embedding, Q/K norms, post norms, GeGLU)."""
    q, kv = heads * head_dim, kv_heads * head_dim
    stream = [0]

    def mat(name, cols, rows, ggml_type):
        stream[0] += 1
        return TensorSpec(name, (cols, rows), ggml_type, "normal", std, stream[0])

    def vec(name, n):
        stream[0] += 1
        return TensorSpec(name, (n,), F32, "ones", std, stream[0])

    tensors = [mat("token_embd.weight", hidden, vocab, embd_type), vec("output_norm.weight", hidden)]
    for l in range(layers):
        p = f"blk.{l}."
        tensors += [vec(p + "attn_norm.weight", hidden), mat(p + "attn_q.weight", hidden, q, wtype),
                    mat(p + "attn_k.weight", hidden, kv, wtype), mat(p + "attn_v.weight", hidden, kv, wtype),
                    vec(p + "attn_q_norm.weight", head_dim), vec(p + "attn_k_norm.weight", head_dim),
                    mat(p + "attn_output.weight", q, hidden, wtype), vec(p + "post_attention_norm.weight", hidden),
                    vec(p + "ffn_norm.weight", hidden), mat(p + "ffn_gate.weight", hidden, ffn, wtype),
                    mat(p + "ffn_up.weight", hidden, ffn, wtype), mat(p + "ffn_down.weight", ffn, hidden, wtype),
                    vec(p + "post_ffw_norm.weight", hidden)]
    md = _arch_metadata("gemma3", layers=layers, hidden=hidden, ffn=ffn, heads=heads, kv_heads=kv_heads,
                        head_dim=head_dim, eps=eps, theta=theta, context=context,
                        extra=[("gemma3.rope.local.freq_base", T_F32V, local_theta),
                               ("gemma3.attention.sliding_window", T_U32, window)])
    return ModelSpec("gemma3", md, tensors, seed=seed)


def _q4km_fallback(name: str, cols: int, ggml_type: int) -> int:
    """Q4_K_M as used here: K-quant blocks need widths that are multiples of 256. A
    narrower matrix falls back to the 32-block type of the same role (Q4_K -> Q4_0,
    Q6_K -> Q8_0), both of which the reference decodes."""
    if cols % 256 == 0:
        return ggml_type
    return {Q4_K: Q4_0, Q5_K: Q8_0, Q6_K: Q8_0}.get(ggml_type, ggml_type)


def baseline_spec(index: int, *, layers: int | None = None) -> ModelSpec:
    """Architectures of the benchmark configurations (index as listed there: 0 tiny llama F32,
    2 Qwen2.5-0.5B, 3 Llama-3-8B, 4 Gemma-3-27B). `layers` trims depth for parity tests."""
    if index == 0:
        s = dense_spec("llama", seed=0, layers=layers or 2, hidden=128, ffn=384, heads=4, kv_heads=2, head_dim=32,
                       vocab=512, eps=1e-5, theta=1e4, wtype=F32, std=0.02)
        s.prompt = uniform_ids(8, 512, seed=0)
        s.description = "tiny llama F32"
        return s
    if index == 2:
        s = dense_spec("qwen2", seed=1, layers=layers or 24, hidden=896, ffn=4864, heads=14, kv_heads=2, head_dim=64,
                       vocab=151936, eps=1e-6, theta=1e6, wtype=Q4_K, embd_type=Q6_K, bias=True, tied=True,
                       type_for=_q4km_fallback)
        s.prompt = uniform_ids(23, 151936, seed=1)
        s.description = "Qwen2.5-0.5B architecture, Q4_K_M"
        return s
    if index == 3:
        s = dense_spec("llama", seed=2, layers=layers or 32, hidden=4096, ffn=14336, heads=32, kv_heads=8, head_dim=128,
                       vocab=128256, eps=1e-5, theta=5e5, wtype=Q4_K, out_type=Q6_K, embd_type=Q6_K)
        s.prompt = uniform_ids(512, 128256, seed=2)
        s.description = "Llama-3-8B architecture, Q4_K_M"
        return s
    if index == 4:
        s = gemma_spec(seed=3, layers=layers or 62, hidden=5376, ffn=21504, heads=32, kv_heads=16, head_dim=128,
                       vocab=262144)
        s.prompt = uniform_ids(1024, 262144, seed=3)
        s.description = "Gemma-3-27B architecture, Q4_K_M"
        return s
    raise ValueError(index)


# ----------------------------------------------- verify-dense.mjs check models

def _lcg(seed: int):
    """verify-dense.mjs:25 — 32-bit LCG returning state / 2^32."""
    state = seed & 0xFFFFFFFF

    def nxt():
        nonlocal state
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        return state / 4294967296.0
    return nxt


def _byte_alphabet() -> list[str]:
    """verify-dense.mjs:54-58 — GPT-2 byte-to-unicode alphabet."""
    kept = [b for b in range(256) if 33 <= b <= 126 or 161 <= b <= 172 or b >= 174]
    codes, extra, out = set(kept), 256, []
    for b in range(256):
        if b in codes:
            out.append(chr(b))
        else:
            out.append(chr(extra))
            extra += 1
    return out


TINY_SPECIALS = ["<|im_start|>", "<|im_end|>", "<|eot_id|>"]


def tiny_dense(kind: str) -> ModelSpec:
    """verify-dense.mjs:60-135: F32 llama/qwen2/qwen3 check models with LCG weights."""
    hidden, heads, kv_heads, head_dim, layers, inter = 64, 4, 2, 16, 2, 128
    tokens = _byte_alphabet() + TINY_SPECIALS
    vocab = len(tokens)
    bias, qk_norm = kind == "qwen2", kind == "qwen3"
    rnd = _lcg({"llama": 7, "qwen2": 11}.get(kind, 13))
    tensors: list[TensorSpec] = []

    def make(name, dims, scale):
        n = int(np.prod(dims))
        vals = np.array([(rnd() * 2 - 1) * scale for _ in range(n)], dtype=np.float32)
        tensors.append(TensorSpec(name, tuple(dims), F32, "lcg", data=vals))

    def eins(name, dims):
        n = int(np.prod(dims))
        vals = np.array([1 + (rnd() * 2 - 1) * 0.1 for _ in range(n)], dtype=np.float32)
        tensors.append(TensorSpec(name, tuple(dims), F32, "lcg", data=vals))

    make("token_embd.weight", [hidden, vocab], 0.6)
    eins("output_norm.weight", [hidden])
    make("output.weight", [hidden, vocab], 0.35)
    for l in range(layers):
        p = f"blk.{l}."
        eins(p + "attn_norm.weight", [hidden])
        make(p + "attn_q.weight", [hidden, heads * head_dim], 0.5)
        make(p + "attn_k.weight", [hidden, kv_heads * head_dim], 0.5)
        make(p + "attn_v.weight", [hidden, kv_heads * head_dim], 0.5)
        make(p + "attn_output.weight", [heads * head_dim, hidden], 0.5)
        if bias:
            make(p + "attn_q.bias", [heads * head_dim], 0.1)
            make(p + "attn_k.bias", [kv_heads * head_dim], 0.1)
            make(p + "attn_v.bias", [kv_heads * head_dim], 0.1)
        if qk_norm:
            eins(p + "attn_q_norm.weight", [head_dim])
            eins(p + "attn_k_norm.weight", [head_dim])
        eins(p + "ffn_norm.weight", [hidden])
        make(p + "ffn_gate.weight", [hidden, inter], 0.45)
        make(p + "ffn_up.weight", [hidden, inter], 0.45)
        make(p + "ffn_down.weight", [inter, hidden], 0.45)
    eos = tokens.index(TINY_SPECIALS[1])
    arch = kind
    md = _arch_metadata(arch, layers=layers, hidden=hidden, ffn=inter, heads=heads, kv_heads=kv_heads,
                        head_dim=head_dim, eps=1e-6, theta=10000.0, context=2048,
                        extra=[("tokenizer.ggml.model", T_STR, "gpt2"), ("tokenizer.ggml.pre", T_STR, "llama-bpe"),
                               ("tokenizer.ggml.eos_token_id", T_U32, eos),
                               ("tokenizer.chat_template", T_STR, "<|im_start|>{{ role }}\n{{ content }}<|im_end|>\n"),
                               ("tokenizer.ggml.tokens", T_ARR, (T_STR, tokens)),
                               ("tokenizer.ggml.token_type", T_ARR, (T_I32, [1 if i < 256 else 3 for i in range(vocab)])),
                               ("tokenizer.ggml.merges", T_ARR, (T_STR, []))])
    spec = ModelSpec(arch, md, tensors, seed=0, description=f"verify-dense tiny-{kind}")
    spec.prompt = tiny_chat([("user", "hello")])
    return spec


def tiny_chat(messages) -> list[int]:
    """verify-dense.mjs:212-220 — chat framing over the byte alphabet (token id = byte)."""
    start, end = 256, 257
    ids: list[int] = []
    for role, content in messages:
        ids += [start, *f"{role}\n".encode(), *content.strip().encode(), end, *b"\n"]
    ids += [start, *b"assistant\n"]
    return ids
