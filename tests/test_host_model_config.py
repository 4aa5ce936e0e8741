"""Host GGUF reader and model configuration, restating tests/model-config.test.ts
(dense cases) and tests/gguf.test.ts of the reference."""
import struct

import numpy as np
import pytest

from webgpu_b200.gguf import GGUF, Tensor, model_config, parse_gguf_header, peek_gguf_header
from webgpu_b200 import synth


def dense_gguf(arch, bias=False, qk_norm=False, gate=True, full_kv=False):
    # model-config.test.ts:10-36
    hidden, heads, kv_heads, head_dim, layers, inter, vocab = 64, 4, 4 if full_kv else 2, 16, 2, 128, 96
    ts = [("token_embd.weight", [hidden, vocab]), ("output_norm.weight", [hidden]), ("output.weight", [hidden, vocab])]
    for l in range(layers):
        p = f"blk.{l}."
        ts += [(p + "attn_norm.weight", [hidden]), (p + "ffn_norm.weight", [hidden]),
               (p + "attn_q.weight", [hidden, heads * head_dim]), (p + "attn_k.weight", [hidden, kv_heads * head_dim]),
               (p + "attn_v.weight", [hidden, kv_heads * head_dim]), (p + "attn_output.weight", [heads * head_dim, hidden])]
        if bias:
            ts += [(p + "attn_q.bias", [heads * head_dim]), (p + "attn_k.bias", [kv_heads * head_dim]),
                   (p + "attn_v.bias", [kv_heads * head_dim])]
        if qk_norm:
            ts += [(p + "attn_q_norm.weight", [head_dim]), (p + "attn_k_norm.weight", [head_dim])]
        if gate:
            ts.append((p + "ffn_gate.weight", [hidden, inter]))
        ts += [(p + "ffn_up.weight", [hidden, inter]), (p + "ffn_down.weight", [inter, hidden])]
    md = {"general.architecture": arch, "general.name": f"{arch} test", f"{arch}.block_count": layers,
          f"{arch}.embedding_length": hidden, f"{arch}.attention.head_count": heads,
          f"{arch}.attention.head_count_kv": kv_heads, f"{arch}.attention.key_length": head_dim,
          f"{arch}.feed_forward_length": inter, f"{arch}.context_length": 8192}
    return GGUF(md, {n: Tensor(n, d, 0, 0, 0, 0) for n, d in ts}, 0, 0)


def test_llama3_dense_decoder_full_context_no_qk_norm():
    c = model_config(dense_gguf("llama"))
    assert (c.family, c.layers, c.heads, c.kv_heads) == ("llama", 2, 4, 2)
    assert (c.head_dim, c.rotary_dim, c.theta, c.attention_scale, c.activation) == (16, 16, 10000, 0.25, "silu")
    assert c.qk_norm is False and c.bias == {"q": False, "k": False, "v": False, "output": False}
    assert c.ffn_gate is True and c.period == 0
    assert c.rope == "norm" and c.sliding_window == 0


def test_rope_scaling_and_sliding_window_from_metadata():
    m = dense_gguf("llama")
    m.metadata.update({"llama.attention.sliding_window": 4096, "llama.rope.scaling.type": "linear",
                       "llama.rope.scaling.factor": 4})
    c = model_config(m)
    assert c.sliding_window == 4096 and c.rope_scale == 0.25
    l31 = dense_gguf("llama")
    l31.metadata.update({"llama.rope.scaling.type": "llama3", "llama.rope.scaling.factor": 8})
    assert model_config(l31).rope_scale == 1
    q = dense_gguf("qwen2")
    q.metadata.update({"qwen2.rope.scaling.type": "linear", "qwen2.rope.scaling.factor": 2})
    assert model_config(q).rope_scale == 0.5


def test_qwen2_bias_and_qwen3_qk_norm_detected():
    q2 = model_config(dense_gguf("qwen2", bias=True))
    assert q2.bias == {"q": True, "k": True, "v": True, "output": False} and q2.qk_norm is False and q2.rope == "neox"
    q3 = model_config(dense_gguf("qwen3", qk_norm=True))
    assert q3.qk_norm is True and q3.rope == "neox" and q3.bias == {"q": False, "k": False, "v": False, "output": False}


def test_ungated_mlp():
    assert model_config(dense_gguf("llama", gate=False)).ffn_gate is False


def test_rejects_moe_bad_shapes_and_missing_tensors():
    moe = dense_gguf("llama")
    moe.tensors["blk.0.ffn_gate_inp.weight"] = Tensor("blk.0.ffn_gate_inp.weight", [64, 4], 0, 0, 0, 0)
    with pytest.raises(ValueError, match="Mixture-of-experts"):
        model_config(moe)
    bad = dense_gguf("llama")
    bad.tensors["blk.1.attn_v.weight"].dims = [64, 64]
    with pytest.raises(ValueError, match="attn_v"):
        model_config(bad)
    missing = dense_gguf("qwen2", bias=True)
    del missing.tensors["blk.1.attn_k.bias"]
    with pytest.raises(ValueError, match=r"attn_k\.bias"):
        model_config(missing)
    nonorm = dense_gguf("llama")
    del nonorm.tensors["blk.1.ffn_norm.weight"]
    with pytest.raises(ValueError, match="ffn_norm"):
        model_config(nonorm)
    with pytest.raises(ValueError, match="Supported text architectures"):
        model_config(dense_gguf("falcon"))


def test_key_length_fallbacks():
    g = dense_gguf("llama", full_kv=True)
    del g.metadata["llama.attention.key_length"]
    del g.metadata["llama.attention.head_count_kv"]
    c = model_config(g)
    assert (c.head_dim, c.kv_heads, c.rotary_dim) == (16, 4, 16)


def header(entries, tensor_count=0):
    # gguf.test.ts:14-21
    out = struct.pack("<IIQQ", 0x46554747, 3, tensor_count, len(entries))
    for key, t, v in entries:
        kb = key.encode()
        out += struct.pack("<Q", len(kb)) + kb + struct.pack("<I", t)
        if t == 8:
            vb = v.encode()
            out += struct.pack("<Q", len(vb)) + vb
        else:
            out += struct.pack("<I", v)
    return out


def test_peek_reports_architecture_name_quantization():
    p = peek_gguf_header(header([("general.architecture", 8, "llama"), ("general.name", 8, "Llama 3.2 1B Instruct"),
                                 ("general.file_type", 4, 15)]))
    assert p == {"architecture": "llama", "name": "Llama 3.2 1B Instruct", "quantization": "Q4_K_M"}


def test_peek_reads_a_small_model_header_through_the_byte_source(tmp_path):
    from webgpu_b200.gguf import peek_gguf
    from webgpu_b200.source import MemorySource, make_source
    data = header([("general.architecture", 8, "qwen3"), ("general.name", 8, "Qwen3 0.6B"), ("general.file_type", 4, 18)])
    p = tmp_path / "qwen3.gguf"
    p.write_bytes(data)
    peek = peek_gguf(make_source(str(p)))
    assert peek["architecture"] == "qwen3" and peek["quantization"] == "Q6_K"
    # a header longer than the first 128 KiB read is found by growing the read
    big = header([("general.description", 8, "x" * 300_000), ("general.architecture", 8, "llama"),
                  ("general.name", 8, "L"), ("general.file_type", 4, 15)])
    assert peek_gguf(MemorySource(np.frombuffer(big, np.uint8)))["quantization"] == "Q4_K_M"
    with pytest.raises(ValueError, match="truncated or invalid"):
        peek_gguf(MemorySource(np.frombuffer(big[:200_000], np.uint8)))


def test_peek_needs_more_bytes_when_truncated():
    full = header([("general.architecture", 8, "qwen2"), ("general.name", 8, "Qwen2.5 0.5B"), ("general.file_type", 4, 12)])
    for cut in (4, 10, 20, len(full) - 1):
        assert peek_gguf_header(full[:cut]) is None


def test_peek_rejects_non_gguf_and_missing_architecture():
    with pytest.raises(ValueError, match="not a GGUF"):
        peek_gguf_header(bytes(64))
    with pytest.raises(ValueError, match="architecture"):
        peek_gguf_header(header([("general.name", 8, "x")]))
    with pytest.raises(ValueError, match="version"):
        peek_gguf_header(struct.pack("<IIQQ", 0x46554747, 9, 0, 0))


@pytest.mark.parametrize("kind", ["llama", "qwen2", "qwen3"])
def test_synthetic_gguf_round_trip(kind):
    spec = synth.tiny_dense(kind)
    image = synth.build_gguf(spec)
    g = parse_gguf_header(image, image.nbytes)
    assert set(g.tensors) == {t.name for t in spec.tensors}
    c = model_config(g)
    assert c.vocab == 259 and c.hidden == 64 and c.rope == ("norm" if kind == "llama" else "neox")
    assert c.bias["q"] == (kind == "qwen2") and c.qk_norm == (kind == "qwen3")
    # tensor bytes land where the directory says
    t = g.tensors["token_embd.weight"]
    vals = image[t.offset:t.offset + t.bytes].view("<f4")
    assert vals[0] == spec.tensors[0].data[0]


def test_baseline_spec_q4km_fallback_types():
    s = synth.baseline_spec(2, layers=1)
    types = {t.name: t.ggml_type for t in s.tensors}
    assert types["token_embd.weight"] == synth.Q8_0  # 896 columns: Q6_K falls back to Q8_0
    assert types["blk.0.attn_q.weight"] == synth.Q4_0
    assert types["blk.0.ffn_down.weight"] == synth.Q4_K  # 4864 = 19 x 256
