"""Pins the oracle's float64 decoder (a C restatement of the reference's
scripts/verify-dense.mjs:138-211 CPU decoder plus its engine rules) against an
independent implementation: HF transformers models run in float64 with the
same weights. The reference's own decoder is JavaScript and cannot run in
this container, and it stores no expected outputs, so this cross-check is the
decoder's pin (the dequant is pinned by the reference's known-answer tests).

The check models are the reference's three verify-dense variants (llama with
adjacent-pair RoPE, qwen2 with Q/K/V bias, qwen3 with Q/K norm). For llama the
Q/K rows are permuted per head so that HF's half-split rotation pairs the same
coordinates the reference's adjacent-pair rotation does; attention scores are
invariant to that permutation."""
import numpy as np
import pytest

import oracle
from webgpu_b200 import synth
from webgpu_b200.gguf import model_config, parse_gguf_header

torch = pytest.importorskip("torch")
transformers = pytest.importorskip("transformers")


def weights_of(spec):
    return {t.name: np.asarray(t.data, np.float64).reshape(tuple(reversed(t.dims))) for t in spec.tensors}


def adjacent_to_half(w, heads, hd):
    """Rows of each head reordered (0,2,4,..,1,3,5,..)."""
    w = w.reshape(heads, hd, -1)
    perm = np.concatenate([np.arange(0, hd, 2), np.arange(1, hd, 2)])
    return w[:, perm, :].reshape(heads * hd, -1)


def hf_model(kind, spec, c):
    W = weights_of(spec)
    common = dict(vocab_size=c.vocab, hidden_size=c.hidden, intermediate_size=c.intermediate, num_hidden_layers=c.layers,
                  num_attention_heads=c.heads, num_key_value_heads=c.kv_heads, head_dim=c.head_dim,
                  rms_norm_eps=c.epsilon, max_position_embeddings=2048, tie_word_embeddings=False,
                  rope_parameters={"rope_type": "default", "rope_theta": c.theta})
    if kind == "llama":
        cfg = transformers.LlamaConfig(**common, attention_bias=False)
        model = transformers.LlamaForCausalLM(cfg)
    elif kind == "qwen2":
        cfg = transformers.Qwen2Config(**common)
        model = transformers.Qwen2ForCausalLM(cfg)
    else:
        cfg = transformers.Qwen3Config(**common, attention_bias=False)
        model = transformers.Qwen3ForCausalLM(cfg)
    model = model.double().eval()
    sd = {}
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    sd["model.embed_tokens.weight"] = T(W["token_embd.weight"])
    sd["model.norm.weight"] = T(W["output_norm.weight"])
    sd["lm_head.weight"] = T(W["output.weight"])
    for l in range(c.layers):
        p, q = f"blk.{l}.", f"model.layers.{l}."
        wq, wk = W[p + "attn_q.weight"], W[p + "attn_k.weight"]
        if kind == "llama":
            wq, wk = adjacent_to_half(wq, c.heads, c.head_dim), adjacent_to_half(wk, c.kv_heads, c.head_dim)
        sd[q + "self_attn.q_proj.weight"] = T(wq)
        sd[q + "self_attn.k_proj.weight"] = T(wk)
        sd[q + "self_attn.v_proj.weight"] = T(W[p + "attn_v.weight"])
        sd[q + "self_attn.o_proj.weight"] = T(W[p + "attn_output.weight"])
        if kind == "qwen2":
            for a in "qkv":
                sd[q + f"self_attn.{a}_proj.bias"] = T(W[p + f"attn_{a}.bias"])
        if kind == "qwen3":
            sd[q + "self_attn.q_norm.weight"] = T(W[p + "attn_q_norm.weight"])
            sd[q + "self_attn.k_norm.weight"] = T(W[p + "attn_k_norm.weight"])
        sd[q + "input_layernorm.weight"] = T(W[p + "attn_norm.weight"])
        sd[q + "post_attention_layernorm.weight"] = T(W[p + "ffn_norm.weight"])
        sd[q + "mlp.gate_proj.weight"] = T(W[p + "ffn_gate.weight"])
        sd[q + "mlp.up_proj.weight"] = T(W[p + "ffn_up.weight"])
        sd[q + "mlp.down_proj.weight"] = T(W[p + "ffn_down.weight"])
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not [m for m in missing if "rotary" not in m], missing
    force_f64(model, c)
    return model


def force_f64(model, c):
    """HF computes RoPE angles and RMS norms in float32 even for float64 models;
    replace both with float64 versions of the same formulas."""
    import types

    def norm_fwd(self, x):
        var = x.pow(2).mean(-1, keepdim=True)
        return self.weight * (x * torch.rsqrt(var + self.variance_epsilon))

    def rope_fwd(self, x, position_ids):
        inv = 1.0 / (c.theta ** (torch.arange(0, c.head_dim, 2, dtype=torch.float64) / c.head_dim))
        freqs = position_ids[..., None].to(torch.float64) * inv
        emb = torch.cat((freqs, freqs), dim=-1)
        return emb.cos().to(x.dtype), emb.sin().to(x.dtype)

    for m in model.modules():
        name = type(m).__name__
        if name.endswith("RMSNorm"):
            m.forward = types.MethodType(norm_fwd, m)
        elif name.endswith("RotaryEmbedding"):
            m.forward = types.MethodType(rope_fwd, m)


@pytest.mark.parametrize("kind", ["llama", "qwen2", "qwen3"])
def test_oracle_decoder_matches_transformers_f64(kind):
    spec = synth.tiny_dense(kind)
    image = synth.build_gguf(spec)
    g = parse_gguf_header(image, image.nbytes)
    c = model_config(g)
    dec = oracle.Decoder(image, g, c, context=256)
    tokens, logits = dec.greedy_decode(spec.prompt, 4)
    model = hf_model(kind, spec, c)
    ids = list(spec.prompt)
    with torch.no_grad():
        for step in range(4):
            out = model(torch.tensor([ids])).logits[0, -1].numpy()
            ref = logits[step]
            err = np.max(np.abs(out - ref)) / np.max(np.abs(ref))
            assert err < 1e-10, (kind, step, err)
            assert int(np.argmax(out)) == tokens[step]
            ids.append(tokens[step])
    dec.close()


def test_oracle_prefill_batches_equal_token_by_token():
    """A prompt fed in one forward or token by token gives the same final logits."""
    spec = synth.baseline_spec(0)
    image = synth.build_gguf(spec)
    g = parse_gguf_header(image, image.nbytes)
    c = model_config(g)
    a = oracle.Decoder(image, g, c, context=256)
    b = oracle.Decoder(image, g, c, context=256)
    la = a.forward(spec.prompt, 0)
    for i, t in enumerate(spec.prompt):
        lb = b.forward([t], i)
    assert np.array_equal(la, lb)
