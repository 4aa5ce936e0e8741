"""Tokenizers and chat framing of the host, mirroring the reference's host code that
turns chat messages into token ids and generated ids back into text:

* `Gpt2Tokenizer` — byte-level BPE over the GPT-2 byte alphabet with ranked merges,
  llama.cpp pre-tokenizer patterns and the Llama 3 / ChatML / Mistral chat framings
  (src/core/gpt2-tokenizer.ts, src/core/bpe.ts of the reference); used for every dense
  family except Gemma (engine.ts:67-69);
* `SentencePieceTokenizer` — SentencePiece BPE by merge scores with UTF-8 byte fallback
  and the Gemma turn framing (src/core/tokenizer.ts);
* `make_tokenizer` picks one by family as the engine does. Models without tokenizer
  metadata (the synthetic benchmark models) get `NoTokenizer`: they are driven by token
  ids (`generate_ids`), and `chat` says why it cannot frame text.

Decoding returns the text of complete UTF-8 sequences only (an unfinished trailing
sequence is withheld, as TextDecoder with stream: true does)."""
from __future__ import annotations

import codecs
import heapq
import math

import regex


def byte_alphabet() -> list[str]:
    """The GPT-2 byte -> printable character table (bpe.ts:2-6): printable Latin-1 bytes map to
    themselves, the other 68 to consecutive code points from 256."""
    printable = set(range(33, 127)) | set(range(161, 173)) | set(range(174, 256))
    out, extra = [], 256
    for b in range(256):
        if b in printable:
            out.append(chr(b))
        else:
            out.append(chr(extra))
            extra += 1
    return out


def merge_symbols(symbols: list[str], score) -> list[str]:
    """Adjacent-pair BPE (bpe.ts:9-38): repeatedly merge the adjacent pair with the highest
    `score(a, b)` (None: not mergeable), ties to the leftmost pair, with a heap of candidate
    pairs invalidated lazily by per-position versions."""
    n = len(symbols)
    if n < 2:
        return list(symbols)
    sym = list(symbols)
    nxt = list(range(1, n)) + [-1]
    prv = list(range(-1, n - 1))
    ver = [0] * n
    heap: list[tuple] = []

    def push(left: int) -> None:
        if left < 0 or nxt[left] < 0:
            return
        right = nxt[left]
        s = score(sym[left], sym[right])
        if s is None or not s > -math.inf:
            return
        heapq.heappush(heap, (-s, left, right, ver[left], ver[right]))

    for i in range(n - 1):
        push(i)
    while heap:
        _, left, right, lv, rv = heapq.heappop(heap)
        if nxt[left] != right or ver[left] != lv or ver[right] != rv:
            continue  # a stale candidate: one side merged since it was queued
        sym[left] += sym[right]
        ver[left] += 1
        ver[right] += 1
        nxt[left] = nxt[right]
        if nxt[right] >= 0:
            prv[nxt[right]] = left
        nxt[right] = -1
        push(prv[left])
        push(left)
    out, i = [], 0
    while i >= 0:
        out.append(sym[i])
        i = nxt[i]
    return out


def _utf8_text(data: bytes) -> str:
    # complete sequences only; invalid bytes become U+FFFD (TextDecoder's default)
    return codecs.getincrementaldecoder("utf-8")("replace").decode(data, final=False)


# llama.cpp's pre-tokenizer patterns by `tokenizer.ggml.pre` name (the same table the
# reference keeps, gpt2-tokenizer.ts:8-20): the split of text into pieces decides which merges
# can apply, so token ids only match with the identical patterns. Unknown names use 'default'.
_CONTRACTION = r"'[sStT]|'[rR][eE]|'[vV][eE]|'[mM]|'[lL][lL]|'[dD]"
_LLAMA3 = (rf"(?:{_CONTRACTION})|[^\r\n\p{{L}}\p{{N}}]?\p{{L}}+|\p{{N}}{{1,3}}| ?[^\s\p{{L}}\p{{N}}]+[\r\n]*|\s*[\r\n]+"
           r"|\s+(?!\S)|\s+")
_PATTERNS = {
    "llama-bpe": _LLAMA3, "llama3": _LLAMA3, "smollm": _LLAMA3, "deepseek-llm": _LLAMA3,
    "qwen2": (rf"(?:{_CONTRACTION})|[^\r\n\p{{L}}\p{{N}}]?\p{{L}}+|\p{{N}}| ?[^\s\p{{L}}\p{{N}}]+[\r\n]*|\s*[\r\n]+"
              r"|\s+(?!\S)|\s+"),
    # qwen35: combining marks (\p{M}) count as letters, so a base letter and its marks stay one piece
    "qwen35": (rf"(?:{_CONTRACTION})|[^\r\n\p{{L}}\p{{N}}]?[\p{{L}}\p{{M}}]+|\p{{N}}| ?[^\s\p{{L}}\p{{M}}\p{{N}}]+[\r\n]*"
               r"|\s*[\r\n]+|\s+(?!\S)|\s+"),
    "gpt2": rf"(?:{_CONTRACTION})| ?\p{{L}}+| ?\p{{N}}+| ?[^\s\p{{L}}\p{{N}}]+|\s+(?!\S)|\s+",
    "default": rf"(?:{_CONTRACTION})| ?\p{{L}}+| ?\p{{N}}+| ?[^\s\p{{L}}\p{{N}}]+|\s+(?!\S)|\s+",
}
_COMPILED: dict[str, regex.Pattern] = {}


def pre_tokenizer(name) -> regex.Pattern:
    key = name if isinstance(name, str) and name in _PATTERNS else "default"
    if key not in _COMPILED:
        _COMPILED[key] = regex.compile(_PATTERNS[key])
    return _COMPILED[key]


def chat_style(metadata: dict, ids: dict) -> str:
    """The chat framing from the GGUF chat template, else from the control tokens the vocabulary
    has (gpt2-tokenizer.ts:32-45), so that a missing template cannot frame a prompt wrongly."""
    template = metadata.get("tokenizer.chat_template")
    if isinstance(template, str):
        for marker, style in (("<|start_header_id|>", "llama3"), ("<|im_start|>", "chatml"), ("[INST]", "mistral")):
            if marker in template:
                return style
    for marker, style in (("<|start_header_id|>", "llama3"), ("<|im_start|>", "chatml"), ("[INST]", "mistral")):
        if marker in ids:
            return style
    raise ValueError("This model does not declare a chat template this runtime understands. Use a chat or instruct "
                     "GGUF (Llama 3, Qwen2/3, Mistral).")


_END_TOKENS = ("<|eot_id|>", "<|eom_id|>", "<|end_of_text|>", "<|im_end|>", "<|endoftext|>", "<|end|>", "</s>",
               "<end_of_turn>")
_CONTROL = 3  # GGUF token type of control tokens


class Gpt2Tokenizer:
    """Byte-level BPE (`tokenizer.ggml.model` = gpt2): Llama 3.x, Qwen2/3, Mistral, SmolLM."""
    usable = True

    def __init__(self, metadata: dict):
        if metadata.get("tokenizer.ggml.model") != "gpt2":
            raise ValueError("This model does not use a byte-level BPE tokenizer.")
        tokens = metadata.get("tokenizer.ggml.tokens")
        merges = metadata.get("tokenizer.ggml.merges")
        if not isinstance(tokens, list) or not isinstance(merges, list) or any(
                not isinstance(m, str) or " " not in m for m in merges):
            raise ValueError("Invalid byte-BPE tokenizer metadata.")
        types = metadata.get("tokenizer.ggml.token_type")
        self.tokens = tokens
        self.types = list(types) if isinstance(types, list) else []
        self.ids = {t: i for i, t in enumerate(tokens)}
        self.ranks = {m: r for r, m in enumerate(merges)}
        self.alphabet = byte_alphabet()
        self.byte_of = {ch: b for b, ch in enumerate(self.alphabet)}
        self.pattern = pre_tokenizer(metadata.get("tokenizer.ggml.pre"))
        self.eos: set[int] = set()
        for key in ("tokenizer.ggml.eos_token_id", "tokenizer.ggml.eot_token_id"):
            v = metadata.get(key)
            if isinstance(v, int) and not isinstance(v, bool) and v >= 0:
                self.eos.add(v)
        many = metadata.get("tokenizer.ggml.eos_token_ids")
        if isinstance(many, list):
            self.eos.update(int(v) for v in many if isinstance(v, int))
        self.eos.update(self.ids[n] for n in _END_TOKENS if n in self.ids)
        self.style = chat_style(metadata, self.ids)

    def encode_text(self, text: str) -> list[int]:
        out: list[int] = []
        for piece in self.pattern.findall(text):
            chars = [self.alphabet[b] for b in piece.encode("utf-8")]
            for symbol in merge_symbols(chars, lambda a, b: -self.ranks[f"{a} {b}"] if f"{a} {b}" in self.ranks else None):
                tid = self.ids.get(symbol)
                if tid is None:
                    raise ValueError("Invalid byte-BPE merge result.")
                out.append(tid)
        return out

    def _control(self, name: str, ids: list[int]) -> None:
        tid = self.ids.get(name)
        ids.extend([tid] if tid is not None else self.encode_text(name))

    def chat(self, messages) -> list[int]:
        ids: list[int] = []
        text = lambda s: ids.extend(self.encode_text(s))  # noqa: E731
        if self.style == "llama3":
            if "<|begin_of_text|>" in self.ids:
                ids.append(self.ids["<|begin_of_text|>"])
            for m in messages:
                self._control("<|start_header_id|>", ids)
                text("assistant" if m["role"] == "assistant" else "user")
                self._control("<|end_header_id|>", ids)
                text("\n\n")
                text(m["content"].strip())
                self._control("<|eot_id|>", ids)
            self._control("<|start_header_id|>", ids)
            text("assistant")
            self._control("<|end_header_id|>", ids)
            text("\n\n")
        elif self.style == "chatml":
            for m in messages:
                self._control("<|im_start|>", ids)
                text(f"{m['role']}\n")
                text(m["content"].strip())
                self._control("<|im_end|>", ids)
                text("\n")
            self._control("<|im_start|>", ids)
            text("assistant\n")
        else:  # mistral
            if "<s>" in self.ids:
                ids.append(self.ids["<s>"])
            for m in messages:
                if m["role"] == "user":
                    self._control("[INST]", ids)
                    text(f" {m['content'].strip()} ")
                    self._control("[/INST]", ids)
                else:
                    text(m["content"].strip())
                    if "</s>" in self.ids:
                        ids.append(self.ids["</s>"])
        return ids

    def decode(self, ids) -> str:
        data = bytearray()
        for i in ids:
            if (self.types[i] if 0 <= i < len(self.types) else 1) == _CONTROL:
                continue
            for ch in self.tokens[i] if 0 <= i < len(self.tokens) else "":
                b = self.byte_of.get(ch)
                if b is not None:
                    data.append(b)
        return _utf8_text(bytes(data))


class SentencePieceTokenizer:
    """SentencePiece BPE by merge score with `<0xHH>` byte fallback (`tokenizer.ggml.model` =
    llama, as Gemma ships it) and the Gemma turn framing."""
    usable = True

    def __init__(self, metadata: dict):
        if metadata.get("tokenizer.ggml.model") != "llama":
            raise ValueError("Only the Gemma SentencePiece tokenizer is supported.")
        tokens, scores = metadata.get("tokenizer.ggml.tokens"), metadata.get("tokenizer.ggml.scores")
        if not isinstance(tokens, list) or not isinstance(scores, list) or len(tokens) != len(scores):
            raise ValueError("Invalid tokenizer metadata.")
        types = metadata.get("tokenizer.ggml.token_type")
        self.tokens, self.scores = tokens, scores
        self.types = list(types) if isinstance(types, list) else []
        self.ids = {t: i for i, t in enumerate(tokens)}
        self.bos = int(metadata.get("tokenizer.ggml.bos_token_id", 2))
        self.eos = {int(metadata.get("tokenizer.ggml.eos_token_id", 1)), self.special("<end_of_turn>")}
        # GGUF's SentencePiece default adds the space prefix unless the model turns it off
        self.prefix = metadata.get("tokenizer.ggml.add_space_prefix") is not False

    def _normal(self, tid: int) -> bool:
        return (self.types[tid] if tid < len(self.types) else 1) == 1

    def special(self, s: str) -> int:
        tid = self.ids.get(s)
        if tid is None:
            raise ValueError(f"Tokenizer lacks {s}.")
        return tid

    def encode_text(self, text: str) -> list[int]:
        chars = ["▁" if c == " " else c for c in ((" " if self.prefix else "") + text)]

        def score(a, b):
            tid = self.ids.get(a + b)
            return self.scores[tid] if tid is not None and self._normal(tid) else None

        out: list[int] = []
        for symbol in merge_symbols(chars, score):
            tid = self.ids.get(symbol)
            if tid is not None and self._normal(tid):
                out.append(tid)
            else:
                out.extend(self.special(f"<0x{b:02X}>") for b in symbol.encode("utf-8"))
        return out

    def chat(self, messages) -> list[int]:
        ids = [self.bos]
        for m in messages:
            ids.append(self.special("<start_of_turn>"))
            role = "model" if m["role"] == "assistant" else "user"
            ids += self.encode_text(f"{role}\n{m['content'].strip()}")
            ids.append(self.special("<end_of_turn>"))
            ids += self.encode_text("\n")
        ids.append(self.special("<start_of_turn>"))
        ids += self.encode_text("model\n")
        return ids

    def decode(self, ids) -> str:
        data = bytearray()
        for i in ids:
            t = self.tokens[i] if 0 <= i < len(self.tokens) else ""
            if len(t) == 6 and t.startswith("<0x") and t.endswith(">") and all(c in "0123456789ABCDEF" for c in t[3:5]):
                data.append(int(t[3:5], 16))
            elif (self.types[i] if 0 <= i < len(self.types) else 1) != _CONTROL:
                data += t.replace("▁", " ").encode("utf-8")
        return _utf8_text(bytes(data))


class NoTokenizer:
    """A model without usable tokenizer metadata: generation by token ids only."""
    usable = False

    def __init__(self, metadata: dict, reason: str):
        self.reason = reason
        eos = metadata.get("tokenizer.ggml.eos_token_id")
        self.eos = {int(eos)} if isinstance(eos, int) else set()

    def chat(self, messages) -> list[int]:
        raise ValueError(f"{self.reason} Drive this model with token ids (generate_ids).")

    def decode(self, ids) -> str:
        return ""


def make_tokenizer(metadata: dict, family: str):
    """engine.ts:67-69 — SentencePiece for Gemma, byte-level BPE for the other dense families."""
    try:
        return SentencePieceTokenizer(metadata) if family == "gemma3" else Gpt2Tokenizer(metadata)
    except ValueError as e:
        return NoTokenizer(metadata, str(e))
