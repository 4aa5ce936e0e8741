"""GGUF header, tensor directory and decoder configuration.

A Python mirror of the reference's src/core/gguf.ts (ahpah-dev/WebGPU 0.9.0):
the same parsing rules, limits and error messages, so the host side of this
runtime accepts and rejects exactly the files the reference does. Line
references below are to that file.
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass, field

# gguf.ts:6-11
QUANTS = {
    0: ("F32", 1, 4), 1: ("F16", 1, 2), 2: ("Q4_0", 32, 18), 8: ("Q8_0", 32, 34),
    12: ("Q4_K", 256, 144), 13: ("Q5_K", 256, 176), 14: ("Q6_K", 256, 210),
}
MAX_SAFE_INTEGER = 2 ** 53 - 1


class NeedMore(Exception):
    """The header continues past the bytes read so far (gguf.ts:12)."""


@dataclass
class Tensor:
    """gguf.ts:4 — dims in GGUF order (dims[0] is the row width)."""
    name: str
    dims: list
    type: int
    offset: int
    bytes: int
    row_bytes: int


@dataclass
class GGUF:
    metadata: dict
    tensors: dict
    data_offset: int
    parameters: int


class _Reader:
    """gguf.ts:13-47."""

    def __init__(self, data: bytes | memoryview):
        self.b = memoryview(data)
        self.offset = 0

    def need(self, n: int):
        if self.offset + n > len(self.b):
            raise NeedMore()

    def u32(self) -> int:
        self.need(4)
        v = struct.unpack_from("<I", self.b, self.offset)[0]
        self.offset += 4
        return v

    def u64(self) -> int:
        self.need(8)
        v = struct.unpack_from("<Q", self.b, self.offset)[0]
        self.offset += 8
        if v > MAX_SAFE_INTEGER:
            raise ValueError("GGUF integer exceeds safe file addressing.")
        return v

    def string(self) -> str:
        n = self.u64()
        if n > 16 * 1024 ** 2:
            raise ValueError("Oversized GGUF string.")
        self.need(n)
        v = bytes(self.b[self.offset:self.offset + n]).decode("utf-8", errors="replace")
        self.offset += n
        return v

    def value(self, vtype: int, depth: int = 0):
        if depth > 2:
            raise ValueError("Invalid nested metadata.")
        if vtype == 8:
            return self.string()
        if vtype == 9:
            t, n = self.u32(), self.u64()
            if n > 2_000_000:
                raise ValueError("Oversized GGUF array.")
            return [self.value(t, depth + 1) for _ in range(n)]
        if vtype == 10:
            return self.u64()
        widths = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 11: 8, 12: 8}
        w = widths.get(vtype)
        if not w:
            raise ValueError(f"Unknown GGUF metadata type {vtype}.")
        self.need(w)
        p = self.offset
        self.offset += w
        fmt = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B", 11: "<q", 12: "<d"}[vtype]
        v = struct.unpack_from(fmt, self.b, p)[0]
        return v != 0 if vtype == 7 else v


def parse_gguf_header(data, file_size: int) -> GGUF:
    """gguf.ts:48-77."""
    r = _Reader(data)
    if r.u32() != 0x46554747:
        raise ValueError("Select a GGUF model file.")
    version = r.u32()
    if version not in (2, 3):
        raise ValueError(f"GGUF version {version} is unsupported.")
    count, kv_count = r.u64(), r.u64()
    if count > 100_000 or kv_count > 100_000:
        raise ValueError("Invalid GGUF counts.")
    metadata = {}
    for _ in range(kv_count):
        key = r.string()
        metadata[key] = r.value(r.u32())
    tensors = {}
    parameters = 0
    for _ in range(count):
        name, nd = r.string(), r.u32()
        if nd < 1 or nd > 4 or name in tensors:
            raise ValueError("Invalid tensor directory.")
        dims = [r.u64() for _ in range(nd)]
        ttype, offset = r.u32(), r.u64()
        q = QUANTS.get(ttype)
        if not q:
            raise ValueError(f"Unsupported tensor quantization {ttype} in {name}. Use Q4_K_M, Q5_K_M, Q6_K or Q8_0.")
        n = math.prod(dims)
        if n > MAX_SAFE_INTEGER or any(d < 1 for d in dims) or dims[0] % q[1] != 0:
            raise ValueError(f"Invalid shape for {name}.")
        row_bytes = dims[0] // q[1] * q[2]
        tensors[name] = Tensor(name, dims, ttype, offset, n // q[1] * q[2], row_bytes)
        parameters += n
    alignment = int(metadata.get("general.alignment", 32))
    if alignment < 1 or alignment > 4096 or (alignment & (alignment - 1)):
        raise ValueError("Invalid GGUF alignment.")
    data_offset = -(-r.offset // alignment) * alignment
    for t in tensors.values():
        t.offset += data_offset
        if t.offset + t.bytes > file_size:
            raise ValueError(f"Truncated model: {t.name}.")
    return GGUF(metadata, tensors, data_offset, parameters)


def read_gguf(source) -> GGUF:
    """gguf.ts:78-83 — grow the header read from 4 MiB until it parses (64 MiB cap)."""
    n = min(source.size, 4 * 1024 ** 2)
    while True:
        try:
            return parse_gguf_header(source.read(0, n), source.size)
        except NeedMore:
            if n >= source.size or n >= 64 * 1024 ** 2:
                raise ValueError("GGUF header exceeds 64 MiB or is truncated.")
            n = min(source.size, n * 2)


DENSE = {"llama", "qwen2", "qwen3"}


@dataclass
class ModelConfig:
    """gguf.ts:87-107."""
    architecture: str
    family: str
    hidden: int
    intermediate: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    epsilon: float
    theta: float
    local_theta: float
    window: int
    period: int
    attention_scale: float
    rope_scale: float
    name: str
    parameters: int
    rotary_dim: int
    max_context: int
    rope: str
    sliding_window: int
    qk_norm: bool = True
    ffn_gate: bool = True
    activation: str = "silu"
    bias: dict = field(default_factory=lambda: {"q": False, "k": False, "v": False, "output": False})
    recurrent: dict | None = None


def _js_number(v):
    try:
        return float(v)
    except (TypeError, ValueError):
        return math.nan


def model_config(g: GGUF) -> ModelConfig:
    """gguf.ts:108-213 (the qwen35 hybrid family is recognised and rejected here:
    its recurrent blocks are outside this runtime's decoder)."""
    raw = g.metadata.get("general.architecture")
    if not isinstance(raw, str) or not raw:
        raise ValueError("The GGUF file has no architecture metadata.")
    arch = raw
    family = "gemma3" if arch == "gemma3" else "qwen35" if arch == "qwen35" else "llama" if arch in DENSE else None
    if not family:
        raise ValueError(f"Supported text architectures: Gemma 3, Llama 3.x and Mistral (llama), Qwen2 and Qwen3. "
                         f"The {arch} architecture is not supported.")
    if family == "qwen35":
        raise ValueError("The qwen35 hybrid recurrent architecture is not supported by this runtime.")

    def num(key, fallback=None):
        v = g.metadata.get(f"{arch}.{key}", fallback)
        v = _js_number(v)
        if not math.isfinite(v) or v <= 0:
            raise ValueError(f"Missing or invalid {arch} metadata: {key}.")
        return v

    def opt(key, fallback):
        return fallback if g.metadata.get(f"{arch}.{key}") is None else num(key)

    layers, hidden, heads = num("block_count"), num("embedding_length"), num("attention.head_count")
    head_dim = opt("attention.key_length", hidden / heads) if family == "llama" else num("attention.key_length")
    embd = g.tensors.get("token_embd.weight")
    cfg = ModelConfig(
        architecture=arch, family=family, hidden=hidden, layers=layers, heads=heads, head_dim=head_dim,
        kv_heads=opt("attention.head_count_kv", heads) if family == "llama" else num("attention.head_count_kv"),
        intermediate=num("feed_forward_length"),
        vocab=embd.dims[1] if embd and len(embd.dims) > 1 else 0,
        epsilon=num("attention.layer_norm_rms_epsilon", 1e-6),
        theta=opt("rope.freq_base", 10_000) if family == "llama" else num("rope.freq_base", 1_000_000),
        local_theta=opt("rope.freq_base", 10_000) if family == "llama" else num("rope.local.freq_base", 10_000),
        window=0 if family == "llama" else num("attention.sliding_window", 1024),
        period=6 if family == "gemma3" else 0,
        attention_scale=1 / math.sqrt(hidden / heads if family == "gemma3" and layers == 62 else head_dim),
        rope_scale=1.0,
        name=str(g.metadata.get("general.name", arch)), parameters=g.parameters,
        rotary_dim=opt("rope.dimension_count", head_dim) if family == "llama" else head_dim,
        max_context=num("context_length", 32768),
        rope="norm" if family == "llama" and arch == "llama" else "neox",
        sliding_window=math.floor(opt("attention.sliding_window", 0)) if family == "llama" else num("attention.sliding_window", 1024),
    )
    if family == "gemma3":
        cfg.activation = "gelu"
    if str(g.metadata.get(f"{arch}.rope.scaling.type", "linear")) == "linear":
        cfg.rope_scale = 1 / num("rope.scaling.factor", 1)
    if float(cfg.max_context) != int(cfg.max_context) or cfg.max_context > MAX_SAFE_INTEGER:
        raise ValueError("Invalid model context length.")

    def is_int(x):
        return float(x) == int(x)

    dims = [layers, hidden, heads, head_dim, cfg.kv_heads, cfg.intermediate, cfg.rotary_dim]
    if (any(not is_int(n) or n < 1 for n in dims) or not is_int(cfg.period) or cfg.period < 0 or heads % cfg.kv_heads
            or head_dim % 2 or cfg.rotary_dim % 2 or cfg.rotary_dim > head_dim or not cfg.vocab or layers > 128
            or heads > 256 or head_dim > 512 or hidden > 16384 or cfg.intermediate > 131072 or cfg.vocab > 1_000_000):
        raise ValueError("Unsupported model dimensions.")
    for k in ("layers", "hidden", "heads", "head_dim", "kv_heads", "intermediate", "rotary_dim", "max_context", "window"):
        setattr(cfg, k, int(getattr(cfg, k)))
    cfg.sliding_window = int(cfg.sliding_window)

    def shape(name, d):
        t = g.tensors.get(name)
        if not t or list(t.dims) != list(d):
            raise ValueError(f"Missing or invalid tensor {name}.")

    hidden, layers, heads, head_dim = cfg.hidden, cfg.layers, cfg.heads, cfg.head_dim
    if family == "llama":
        if "blk.0.ffn_gate_inp.weight" in g.tensors or "blk.0.ffn_gate_exps.weight" in g.tensors:
            raise ValueError("Mixture-of-experts models are not supported.")
        cfg.ffn_gate = "blk.0.ffn_gate.weight" in g.tensors
        cfg.qk_norm = "blk.0.attn_q_norm.weight" in g.tensors
        for key in ("q", "k", "v", "output"):
            cfg.bias[key] = f"blk.0.attn_{key}.bias" in g.tensors
        attn, kv = heads * head_dim, cfg.kv_heads * head_dim
        shape("token_embd.weight", [hidden, cfg.vocab])
        shape("output_norm.weight", [hidden])
        if "output.weight" in g.tensors:
            shape("output.weight", [hidden, cfg.vocab])
        for l in range(layers):
            p = f"blk.{l}."
            shape(p + "attn_norm.weight", [hidden])
            shape(p + "ffn_norm.weight", [hidden])
            shape(p + "attn_q.weight", [hidden, attn])
            shape(p + "attn_k.weight", [hidden, kv])
            shape(p + "attn_v.weight", [hidden, kv])
            shape(p + "attn_output.weight", [attn, hidden])
            if cfg.bias["q"]:
                shape(p + "attn_q.bias", [attn])
            if cfg.bias["k"]:
                shape(p + "attn_k.bias", [kv])
            if cfg.bias["v"]:
                shape(p + "attn_v.bias", [kv])
            if cfg.bias["output"]:
                shape(p + "attn_output.bias", [hidden])
            if cfg.qk_norm:
                for key in ("attn_q_norm", "attn_k_norm"):
                    shape(p + key + ".weight", [head_dim])
            if cfg.ffn_gate:
                shape(p + "ffn_gate.weight", [hidden, cfg.intermediate])
            shape(p + "ffn_up.weight", [hidden, cfg.intermediate])
            shape(p + "ffn_down.weight", [cfg.intermediate, hidden])
        return cfg
    shape("token_embd.weight", [hidden, cfg.vocab])
    shape("output_norm.weight", [hidden])
    if "output.weight" in g.tensors:
        shape("output.weight", [hidden, cfg.vocab])
    for l in range(layers):
        p = f"blk.{l}."
        for key in ("attn_norm", "post_attention_norm", "ffn_norm", "post_ffw_norm"):
            shape(p + key + ".weight", [hidden])
        for key in ("attn_q_norm", "attn_k_norm"):
            shape(p + key + ".weight", [head_dim])
        shape(p + "attn_q.weight", [hidden, heads * head_dim])
        for key in ("attn_k", "attn_v"):
            shape(p + key + ".weight", [hidden, cfg.kv_heads * head_dim])
        shape(p + "attn_output.weight", [heads * head_dim, hidden])
        for key in ("ffn_gate", "ffn_up"):
            shape(p + key + ".weight", [hidden, cfg.intermediate])
        shape(p + "ffn_down.weight", [cfg.intermediate, hidden])
    return cfg


# gguf.ts:222-241
FILE_TYPES = {0: "F32", 1: "F16", 2: "Q4_0", 3: "Q4_1", 7: "Q8_0", 8: "Q5_0", 9: "Q5_1", 10: "Q2_K", 11: "Q3_K_S",
              12: "Q3_K_M", 13: "Q3_K_L", 14: "Q4_K_S", 15: "Q4_K_M", 16: "Q5_K_S", 17: "Q5_K_M", 18: "Q6_K", 19: "Q8_K"}


def peek_gguf_header(data):
    """gguf.ts:242-248 — architecture, name and quantization label, or None if more bytes are needed."""
    try:
        r = _Reader(data)
        if r.u32() != 0x46554747:
            raise ValueError("This file is not a GGUF model.")
        version = r.u32()
        if version not in (2, 3):
            raise ValueError(f"GGUF version {version} is unsupported.")
        r.u64()
        count = r.u64()
        if count > 100_000:
            raise ValueError("Invalid GGUF counts.")
        found = {}
        for _ in range(min(count, 512)):
            key = r.string()
            if key in ("general.architecture", "general.name", "general.file_type"):
                found[key] = r.value(r.u32())
            else:
                t = r.u32()
                if t == 9:
                    r.u32()
                    n = r.u64()
                    if n > 2_000_000:
                        raise ValueError("Oversized GGUF array.")
                    for _ in range(n):
                        r.value(r.u32(), 1)
                else:
                    r.value(t)
            if all(k in found for k in ("general.architecture", "general.name", "general.file_type")):
                break
        arch = str(found.get("general.architecture", ""))
        if not arch:
            raise ValueError("The GGUF file has no architecture metadata.")
        ft = found.get("general.file_type")
        return {"architecture": arch, "name": str(found.get("general.name", "")),
                "quantization": FILE_TYPES.get(int(ft), "") if ft is not None else ""}
    except NeedMore:
        return None


def peek_gguf(source) -> dict:
    """gguf.ts:242-248 — reads the header through a byte source, doubling the read from 128 KiB
    until the architecture, name and quantization label parse (8 MiB at most)."""
    n = min(source.size, 128 * 1024)
    while True:
        peek = peek_gguf_header(bytes(source.read(0, n)))
        if peek:
            return peek
        if n >= source.size or n >= 8 * 1024 ** 2:
            raise ValueError("The GGUF header is truncated or invalid.")
        n = min(source.size, n * 2)


def to_native_config(c: ModelConfig):
    """ModelConfig -> wgd_model_config."""
    from ._native import ModelConfigC
    return ModelConfigC(
        family=1 if c.family == "gemma3" else 0, hidden=c.hidden, intermediate=c.intermediate, layers=c.layers,
        heads=c.heads, kv_heads=c.kv_heads, head_dim=c.head_dim, vocab=c.vocab, epsilon=c.epsilon, theta=c.theta,
        local_theta=c.local_theta, window=c.window, period=c.period, attention_scale=c.attention_scale,
        rope_scale=c.rope_scale, rotary_dim=c.rotary_dim, rope_mode=1 if c.rope == "norm" else 0,
        sliding_window=c.sliding_window, qk_norm=int(c.qk_norm), ffn_gate=int(c.ffn_gate),
        activation=1 if c.activation == "gelu" else 0, bias_q=int(c.bias["q"]), bias_k=int(c.bias["k"]),
        bias_v=int(c.bias["v"]), bias_output=int(c.bias["output"]))
