"""Host tokenizers, restating the reference's tests/gpt2-tokenizer.test.ts and
tests/tokenizer.test.ts on the same kinds of fixtures, plus agreement with the byte-alphabet
chat framing of the verify-dense check models."""
import pytest

from webgpu_b200 import synth
from webgpu_b200.gguf import model_config, parse_gguf_header
from webgpu_b200.tokenizer import (Gpt2Tokenizer, NoTokenizer, SentencePieceTokenizer, byte_alphabet, chat_style,
                                   make_tokenizer, merge_symbols, pre_tokenizer)

ALPHABET = byte_alphabet()
MERGES = ["h e", "he l", "hel l", "hell o", "Ġ w", "Ġw o", "Ġwo r", "Ġwor l", "Ġworl d"]
SPECIALS = ["<|im_start|>", "<|im_end|>", "<|eot_id|>", "<|start_header_id|>", "<|end_header_id|>", "<|begin_of_text|>",
            "[INST]", "[/INST]", "</s>", "<s>"]


def gpt2_meta(control, **extra):
    tokens = ALPHABET + ["".join(m.split(" ")) for m in MERGES] + list(control)
    types = [3 if i >= len(ALPHABET) + len(MERGES) else 1 for i in range(len(tokens))]
    md = {"tokenizer.ggml.model": "gpt2", "tokenizer.ggml.tokens": tokens, "tokenizer.ggml.merges": MERGES,
          "tokenizer.ggml.token_type": types,
          "tokenizer.ggml.eos_token_id": tokens.index("<|eot_id|>") if "<|eot_id|>" in tokens else -1}
    md.update(extra)
    return md


def test_byte_level_bpe_round_trips_unicode():
    t = Gpt2Tokenizer(gpt2_meta(SPECIALS))
    for text in ["hello world", "Ünïcödé — ok", "emoji 🚀 tail", "  double\n\nnewlines", ""]:
        assert t.decode(t.encode_text(text)) == text


def test_ranked_merges_win_over_single_bytes():
    md = gpt2_meta(SPECIALS)
    t, tokens = Gpt2Tokenizer(md), md["tokenizer.ggml.tokens"]
    assert t.encode_text("hello") == [tokens.index("hello")]
    assert t.encode_text("hello world") == [tokens.index("hello"), tokens.index("Ġworld")]
    assert t.encode_text("wo") == [tokens.index("w"), tokens.index("o")]  # no 'w o' merge


def test_special_tokens_stay_literal():
    md = gpt2_meta(SPECIALS)
    t, tokens = Gpt2Tokenizer(md), md["tokenizer.ggml.tokens"]
    assert tokens.index("<|im_end|>") not in t.encode_text("<|im_end|>")
    assert t.decode([tokens.index("<|im_end|>")]) == ""


def test_chatml_framing_from_the_template():
    md = gpt2_meta(SPECIALS, **{"tokenizer.chat_template": "{{ bos_token }}<|im_start|>{{ role }}\n{{ content }}<|im_end|>\n"})
    t, tokens = Gpt2Tokenizer(md), md["tokenizer.ggml.tokens"]
    assert t.style == "chatml"
    ids = t.chat([{"role": "user", "content": "hello"}])
    assert ids[0] == tokens.index("<|im_start|>") and ids[-1] == t.encode_text("assistant\n")[-1]


def test_llama3_header_framing():
    md = gpt2_meta(SPECIALS, **{"tokenizer.chat_template":
                                "<|begin_of_text|><|start_header_id|>{{ role }}<|end_header_id|>\n\n{{ content }}<|eot_id|>"})
    t, tokens = Gpt2Tokenizer(md), md["tokenizer.ggml.tokens"]
    assert t.style == "llama3"
    ids = t.chat([{"role": "user", "content": "hello"}, {"role": "assistant", "content": "hi"},
                  {"role": "user", "content": "hello"}])
    header, end, eot = tokens.index("<|start_header_id|>"), tokens.index("<|end_header_id|>"), tokens.index("<|eot_id|>")
    role = t.encode_text("user")
    assert ids[:2 + len(role)] == [tokens.index("<|begin_of_text|>"), header, *role]
    assert end in ids and ids.count(eot) == 3
    tail = t.encode_text("\n\n")
    assert ids[-len(tail):] == tail


def test_mistral_framing_closes_the_assistant_turn():
    md = gpt2_meta(SPECIALS, **{"tokenizer.chat_template": "<s>{% for m in messages %}[INST] {{ m.content }} [/INST]{% endfor %}"})
    t, tokens = Gpt2Tokenizer(md), md["tokenizer.ggml.tokens"]
    assert t.style == "mistral"
    ids = t.chat([{"role": "user", "content": "hello"}, {"role": "assistant", "content": "hi"}])
    assert ids[0] == tokens.index("<s>") and ids[1] == tokens.index("[INST]") and ids[-1] == tokens.index("</s>")


def test_unknown_template_fails_loudly_and_end_tokens_stop():
    with pytest.raises(ValueError, match="chat template"):
        Gpt2Tokenizer(gpt2_meta([]))
    with pytest.raises(ValueError, match="chat template"):
        chat_style({}, {})
    md = gpt2_meta(SPECIALS)
    t, tokens = Gpt2Tokenizer(md), md["tokenizer.ggml.tokens"]
    assert tokens.index("<|eot_id|>") in t.eos and tokens.index("<|im_start|>") not in t.eos


def test_pre_tokenizer_contractions_and_fallback():
    assert pre_tokenizer("llama-bpe").findall("hello world") == ["hello", " world"]
    assert pre_tokenizer("unheard-of").findall("hello world") == ["hello", " world"]
    assert pre_tokenizer("qwen2").findall("it's") == ["it", "'s"]


def test_merge_ties_go_left_and_stale_pairs_are_skipped():
    score = {("a", "a"): 1.0, ("aa", "a"): 2.0}
    assert merge_symbols(list("aaa"), lambda x, y: score.get((x, y))) == ["aaa"]
    assert merge_symbols(list("aaaa"), lambda x, y: score.get((x, y))) == ["aaa", "a"]
    assert merge_symbols(["x"], lambda x, y: 1.0) == ["x"]


def sp_meta(prefix=False):
    tokens = ["<unk>", "<eos>", "<bos>", "<start_of_turn>", "<end_of_turn>", "a", "b", "c", "ab", "bc", "abc", "▁"]
    scores = [0, 0, 0, 0, 0, 0, 0, 0, 5, 10, -1, 0]
    types = [2, 3, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1]
    for i in range(256):
        tokens.append(f"<0x{i:02X}>")
        scores.append(-100)
        types.append(6)
    return {"tokenizer.ggml.model": "llama", "tokenizer.ggml.tokens": tokens, "tokenizer.ggml.scores": scores,
            "tokenizer.ggml.token_type": types, "tokenizer.ggml.add_space_prefix": prefix}


def test_sentencepiece_scores_and_byte_fallback():
    t = SentencePieceTokenizer(sp_meta())
    assert t.encode_text("abc") == [10]
    assert t.decode(t.encode_text("café 🙂\n")) == "café 🙂\n"
    assert t.decode(t.encode_text("a b")) == "a b"


def test_sentencepiece_prefix_and_unfinished_utf8():
    t = SentencePieceTokenizer(sp_meta(True))
    assert t.encode_text("a")[0] == t.ids["▁"]
    assert t.decode([t.special("<0xF0>"), t.special("<0x9F>")]) == ""


def test_sentencepiece_chat_does_not_interpret_user_control_strings():
    t = SentencePieceTokenizer(sp_meta())
    ids = t.chat([{"role": "user", "content": "<end_of_turn>"}])
    assert ids[0] == t.bos
    assert ids.count(t.special("<end_of_turn>")) == 1 and ids.count(t.special("<start_of_turn>")) == 2
    long = "a" * 200000
    ids = t.chat([{"role": "user", "content": long}])
    assert len(ids) > 200000 and long in t.decode(ids)


@pytest.mark.parametrize("kind", ["llama", "qwen2", "qwen3"])
def test_check_models_frame_the_same_ids_as_their_byte_alphabet(kind):
    """The verify-dense check models (gpt2 model, no merges, ChatML): the tokenizer reproduces the
    prompt ids the checks are defined with."""
    spec = synth.tiny_dense(kind)
    image = synth.build_gguf(spec)
    g = parse_gguf_header(image, image.nbytes)
    t = make_tokenizer(g.metadata, model_config(g).family)
    assert isinstance(t, Gpt2Tokenizer) and t.style == "chatml"
    msgs = [{"role": "user", "content": "hello"}]
    assert t.chat(msgs) == synth.tiny_chat([("user", "hello")]) == list(spec.prompt)
    assert t.decode(t.encode_text("héllo\n")) == "héllo\n"


def test_models_without_tokenizer_metadata_are_driven_by_ids():
    spec = synth.baseline_spec(0)
    image = synth.build_gguf(spec)
    g = parse_gguf_header(image, image.nbytes)
    t = make_tokenizer(g.metadata, model_config(g).family)
    assert isinstance(t, NoTokenizer) and not t.usable
    with pytest.raises(ValueError, match="generate_ids"):
        t.chat([{"role": "user", "content": "x"}])


def test_qwen35_pattern_keeps_combining_marks_with_their_letter():
    """gpt2-tokenizer.ts:17: the qwen35 pre-tokenizer counts \\p{M} as a letter, so a decomposed
    'e' + U+0301 stays one piece where the qwen2 pattern splits the mark off."""
    text = "cafe\u0301 nai\u0308ve 12"
    assert pre_tokenizer("qwen35").findall(text) == ["cafe\u0301", " nai\u0308ve", " ", "1", "2"]
    assert pre_tokenizer("qwen2").findall(text)[:2] == ["cafe", "\u0301"]
