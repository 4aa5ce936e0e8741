"""CPU oracle (TEST INFRASTRUCTURE ONLY): ctypes binding of oracle/oracle.c.

Only the tests, the smoke check and the CPU-baseline leg of bench.py use this
package, and only as the checker / the timed CPU restatement. The product path
(webgpu_b200) never imports it.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None


class OracleConfig(ctypes.Structure):
    _fields_ = [("family", ctypes.c_int32), ("hidden", ctypes.c_int32), ("intermediate", ctypes.c_int32),
                ("layers", ctypes.c_int32), ("heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("vocab", ctypes.c_int32), ("epsilon", ctypes.c_double),
                ("theta", ctypes.c_double), ("local_theta", ctypes.c_double), ("window", ctypes.c_int32),
                ("period", ctypes.c_int32), ("attention_scale", ctypes.c_double), ("rope_scale", ctypes.c_double),
                ("rotary_dim", ctypes.c_int32), ("rope_mode", ctypes.c_int32), ("sliding_window", ctypes.c_int32),
                ("qk_norm", ctypes.c_int32), ("ffn_gate", ctypes.c_int32), ("activation", ctypes.c_int32),
                ("bias_q", ctypes.c_int32), ("bias_k", ctypes.c_int32), ("bias_v", ctypes.c_int32),
                ("bias_output", ctypes.c_int32), ("context", ctypes.c_int32)]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"oracle not built: {LIB_PATH} (make -C oracle)")
        L = ctypes.CDLL(LIB_PATH)
        vp, i64, d = ctypes.c_void_p, ctypes.c_int64, ctypes.c_double
        L.or_half_to_float.restype = d
        L.or_half_to_float.argtypes = [ctypes.c_uint32]
        L.or_decode_weight.restype = d
        L.or_decode_weight.argtypes = [vp, ctypes.c_int, i64]
        L.or_decode_weight_f32.restype = ctypes.c_float
        L.or_decode_weight_f32.argtypes = [vp, ctypes.c_int, i64]
        L.or_dequant.argtypes = [vp, ctypes.c_int, i64, vp]
        L.or_dequant_f32.argtypes = [vp, ctypes.c_int, i64, vp]
        L.or_matmul.argtypes = [vp, ctypes.c_int, i64, i64, vp, ctypes.c_int, i64, i64, ctypes.c_int, vp]
        L.or_greedy.restype = i64
        L.or_greedy.argtypes = [vp, i64]
        L.or_greedy_f64.restype = i64
        L.or_greedy_f64.argtypes = [vp, i64]
        L.or_sample.restype = i64
        L.or_sample.argtypes = [vp, i64, d, ctypes.c_int, d, d]
        L.or_set_threads.argtypes = [ctypes.c_int]
        L.or_rmsnorm.argtypes = [vp, vp, i64, i64, d, vp]
        L.or_rope.argtypes = [vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, d, d, d, ctypes.c_int,
                              ctypes.c_int, ctypes.c_int, vp]
        L.or_attention.argtypes = [vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, d,
                                   ctypes.c_int, ctypes.c_int, vp]
        L.or_model_create.restype = vp
        L.or_model_create.argtypes = [ctypes.POINTER(OracleConfig)]
        L.or_model_destroy.argtypes = [vp]
        L.or_model_set.restype = ctypes.c_int
        L.or_model_set.argtypes = [vp, ctypes.c_char_p, vp, ctypes.c_int, i64, i64]
        L.or_state_create.restype = vp
        L.or_state_create.argtypes = [vp, ctypes.c_int]
        L.or_state_destroy.argtypes = [vp, vp]
        L.or_state_fill.restype = ctypes.c_int
        L.or_state_fill.argtypes = [vp, vp, ctypes.c_int, ctypes.c_uint64]
        L.or_forward.restype = ctypes.c_int
        L.or_forward.argtypes = [vp, vp, vp, ctypes.c_int, ctypes.c_int, vp]
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def half_to_float(h: int) -> float:
    return lib().or_half_to_float(h)


def decode(data: np.ndarray, ggml_type: int, n: int) -> np.ndarray:
    """quant.ts decodeWeight over the first n elements, f64."""
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.empty(n, np.float64)
    lib().or_dequant(_ptr(data), ggml_type, n, _ptr(out))
    return out


def decode_f32(data: np.ndarray, ggml_type: int, n: int) -> np.ndarray:
    """WGSL-order fp32 twin of decodeWeight."""
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.empty(n, np.float32)
    lib().or_dequant_f32(_ptr(data), ggml_type, n, _ptr(out))
    return out


def matmul(w: np.ndarray, ggml_type: int, rows: int, cols: int, x: np.ndarray, batch: int, threads: int = 8) -> np.ndarray:
    """y[b, r] = sum_c decode(W)[r, c] * x[b, c] in f64 (verify.ts:32-35)."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty((batch, rows), np.float64)
    lib().or_set_threads(threads)
    lib().or_matmul(_ptr(w), ggml_type, rows, cols, _ptr(x), batch, rows, 0, 0, _ptr(y))
    return y


def greedy(logits: np.ndarray) -> int:
    a = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().or_greedy(_ptr(a), a.size))


def sample(logits: np.ndarray, temperature: float, top_k: int, top_p: float, uniform: float) -> int:
    """engine.ts:305-324 with Math.random() replaced by `uniform`; -1 when no logit is finite."""
    a = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().or_sample(_ptr(a), a.size, float(temperature), int(top_k), float(top_p), float(uniform)))


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    n = w.size
    y = np.empty(x.shape, np.float64)
    lib().or_rmsnorm(_ptr(x), _ptr(w), n, x.size // n, eps, _ptr(y))
    return y


def rope(x, w, n, heads, hd, start, theta, scale, eps, rot, mode, qk_norm) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    wa = np.ascontiguousarray(w, np.float32) if w is not None else None
    y = np.empty(x.size, np.float64)
    lib().or_rope(_ptr(x), _ptr(wa) if wa is not None else None, n, heads, hd, start, theta, scale, eps, rot, mode,
                  int(qk_norm), _ptr(y))
    return y


def attention(q, k, v, n, heads, kv_heads, hd, start, scale, window, capacity) -> np.ndarray:
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    y = np.empty(n * heads * hd, np.float64)
    lib().or_attention(_ptr(q), _ptr(k), _ptr(v), n, heads, kv_heads, hd, start, scale, window, capacity, _ptr(y))
    return y


class Decoder:
    """The float64 CPU decoder over a GGUF image (verify-dense.mjs:138-211 plus the
    engine's block rules). `image` must stay alive while the decoder is used."""

    def __init__(self, image: np.ndarray, gguf, config, context: int, threads: int = 1):
        L = lib()
        c = config
        self.image = image
        self.config = c
        cfg = OracleConfig(
            family=1 if c.family == "gemma3" else 0, hidden=c.hidden, intermediate=c.intermediate, layers=c.layers,
            heads=c.heads, kv_heads=c.kv_heads, head_dim=c.head_dim, vocab=c.vocab, epsilon=c.epsilon, theta=c.theta,
            local_theta=c.local_theta, window=c.window, period=c.period, attention_scale=c.attention_scale,
            rope_scale=c.rope_scale, rotary_dim=c.rotary_dim, rope_mode=1 if c.rope == "norm" else 0,
            sliding_window=c.sliding_window, qk_norm=int(c.qk_norm), ffn_gate=int(c.ffn_gate),
            activation=1 if c.activation == "gelu" else 0, bias_q=int(c.bias["q"]), bias_k=int(c.bias["k"]),
            bias_v=int(c.bias["v"]), bias_output=int(c.bias["output"]), context=context)
        self._cfg = cfg
        self.model = L.or_model_create(ctypes.byref(cfg))
        base = image.ctypes.data
        for t in gguf.tensors.values():
            rows = t.bytes // t.row_bytes
            L.or_model_set(self.model, t.name.encode(), ctypes.c_void_p(base + t.offset), t.type, t.dims[0], rows)
        self.state = L.or_state_create(self.model, context)
        L.or_set_threads(threads)

    def forward(self, ids, start: int) -> np.ndarray:
        n = len(ids)
        arr = np.asarray(ids, dtype=np.int32)
        logits = np.empty(self.config.vocab, np.float64)
        if lib().or_forward(self.model, self.state, _ptr(arr), n, start, _ptr(logits)) != 0:
            raise ValueError("oracle forward: bad arguments")
        return logits

    def fill_cache(self, n: int, seed: int = 1) -> None:
        """Benchmark support: K/V rows of positions [0, n) set to seeded values, so that timing
        can decode at position n without first running an n-token prompt (not for parity)."""
        if lib().or_state_fill(self.model, self.state, n, seed) != 0:
            raise ValueError("fill_cache: n exceeds the context")

    def greedy_decode(self, prompt, steps: int, batch: int | None = None):
        """Prefill the prompt, then greedy-decode `steps` tokens. Returns (tokens, logits list)."""
        logits = self.forward(list(prompt), 0)
        tokens, all_logits = [], [logits]
        pos = len(prompt)
        for i in range(steps):
            tok = int(np.argmax(np.where(np.isfinite(logits), logits, -np.inf)))
            tokens.append(tok)
            if i + 1 < steps:
                logits = self.forward([tok], pos)
                all_logits.append(logits)
                pos += 1
        return tokens, all_logits

    def close(self):
        if self.model:
            lib().or_state_destroy(self.state, self.model)
            lib().or_model_destroy(self.model)
            self.model = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
