"""Prompt text side of the pipeline: the s2.cpp-compatible BPE tokenizer and
the Dual-AR prompt builder (host code; the GPU path starts at the prompt
tensor).

* `S2Tokenizer` restates `S2CppBpeTokenizer` (crates/fish_s2_infer/src/
  tokenizer_s2cpp.rs:1-249) and the special ids of `S2Tokenizer`
  (tokenizer.rs:28-96): vocab and merges from a tokenizer.json, special
  tokens matched longest first, whitespace-led pre-tokenization, GPT-2
  byte-level symbols, lowest-rank merge first.
* `build_prompt` restates prompt.rs:105-220: the (num_codebooks + 1) x cols
  prompt tensor with the system / user / assistant turns in row 0 and, with
  a reference clip, its codes (semantic ids offset by semantic_begin_id in
  row 0, the codebooks in rows 1..).
* `load_prompt_codes` reads the reference's prompt-codes JSON
  (prompt.rs:22-60).
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Optional

import numpy as np

from .s2d import PromptTensor, S2dError

NEWLINE_TOKEN_ID = 198  # tokenizer.rs:9: Qwen's newline id, which s2.cpp uses as is


def bytes_to_unicode() -> dict[int, str]:
    """The GPT-2 byte-level alphabet (tokenizer.rs:98 gpt2_byte_to_unicode):
    printable Latin-1 bytes map to themselves, the other 68 bytes to
    U+0100 onwards in byte order."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAD)) + list(range(0xAE, 0x100))
    table, n = {}, 0
    for b in range(256):
        if b in keep:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + n)
            n += 1
    return table


_BYTE_TABLE = bytes_to_unicode()


def bytelevel(text: str) -> str:
    return "".join(_BYTE_TABLE[b] for b in text.encode("utf-8"))


def _utf8_chars(text: str) -> list[str]:
    """tokenizer_s2cpp.rs:227: characters by their UTF-8 lead bytes."""
    return list(text)


def _pre_tokenize(text: str) -> list[str]:
    """tokenizer_s2cpp.rs:203: a space, tab, CR or LF starts a new word and
    stays at its front."""
    words, cur = [], ""
    for ch in _utf8_chars(text):
        if ch in (" ", "\t", "\n", "\r"):
            if cur:
                words.append(cur)
            cur = ch
            continue
        cur += ch
    if cur:
        words.append(cur)
    return words


@dataclass
class TokenizerConfig:  # tokenizer.rs:20
    im_start_id: int
    im_end_id: int
    voice_id: int


class S2Tokenizer:
    """tokenizer_s2cpp.rs S2CppBpeTokenizer + tokenizer.rs S2Tokenizer."""

    def __init__(self, vocab: dict[str, int], merges: list[tuple[str, str]], specials: list[tuple[str, int]]):
        self.vocab = vocab
        self.merge_rank = {a + b: r for r, (a, b) in enumerate(merges)}
        self.specials = sorted(specials, key=lambda s: -len(s[0].encode("utf-8")))
        self.config = TokenizerConfig(self._special("<|im_start|>"), self._special("<|im_end|>"),
                                      self._special("<|voice|>"))

    @classmethod
    def from_json_bytes(cls, data: bytes) -> "S2Tokenizer":
        """tokenizer_s2cpp.rs:45-96: added tokens first (special ones also
        matched in text), then the model vocab where not already present, and
        merges as pairs or "a b" lines."""
        try:
            doc = json.loads(data)
        except ValueError as e:
            raise S2dError(-1, f"parse tokenizer json: {e}") from None
        vocab, specials = {}, []
        for tok in doc.get("added_tokens") or []:
            if not tok.get("content"):
                continue
            vocab[tok["content"]] = int(tok["id"])
            if tok.get("special", False):
                specials.append((tok["content"], int(tok["id"])))
        merges = []
        model = doc.get("model") or {}
        for k, v in (model.get("vocab") or {}).items():
            vocab.setdefault(k, int(v))
        for m in model.get("merges") or []:
            if isinstance(m, str):
                if " " not in m:
                    raise S2dError(-1, "invalid merge line")
                a, b = m.split(" ", 1)
            else:
                a, b = m
            merges.append((a, b))
        return cls(vocab, merges, specials)

    @classmethod
    def from_file(cls, path) -> "S2Tokenizer":
        try:
            data = Path(path).read_bytes()
        except OSError as e:
            raise S2dError(-2, f"read tokenizer: {e}") from None
        return cls.from_json_bytes(data)

    def _special(self, token: str) -> int:
        if token not in self.vocab:
            raise S2dError(-1, f"missing special token id for {token!r}")
        return self.vocab[token]

    def token_to_id(self, token: str) -> Optional[int]:
        return self.vocab.get(token)

    def encode_newline(self) -> list[int]:
        return [NEWLINE_TOKEN_ID]

    def encode_s2cpp(self, text: str) -> list[int]:
        """tokenizer_s2cpp.rs:98-116."""
        ids = []
        for segment, special in self._split_on_specials(text):
            if special is not None:
                ids.append(special)
            elif segment:
                for word in _pre_tokenize(segment):
                    ids.extend(self._bpe_word(word))
        return ids

    def _split_on_specials(self, text: str):
        """tokenizer_s2cpp.rs:146-201: every occurrence of every special token,
        sorted by position (longer first at one position), overlaps dropped."""
        matches = []
        for tok, tid in self.specials:
            pos = 0
            while True:
                found = text.find(tok, pos)
                if found < 0:
                    break
                matches.append((found, len(tok), tid))
                pos = found + len(tok)
        matches.sort(key=lambda m: (m[0], -m[1]))
        out, last, pos = [], 0, 0
        for p, n, tid in matches:
            if p < last:
                continue
            last = p + n
            if p > pos:
                out.append((text[pos:p], None))
            out.append((text[p:p + n], tid))
            pos = p + n
        if pos < len(text):
            out.append((text[pos:], None))
        return out

    def _bpe_word(self, word: str) -> list[int]:
        """tokenizer_s2cpp.rs:118-144: the whole byte-level word if it is in
        the vocab, else merge the adjacent pair of lowest rank (the first on
        ties) until none applies; symbols outside the vocab are dropped."""
        bl = bytelevel(word)
        if bl in self.vocab:
            return [self.vocab[bl]]
        sym = list(bl)
        while len(sym) > 1:
            best, at = None, -1
            for i in range(len(sym) - 1):
                r = self.merge_rank.get(sym[i] + sym[i + 1])
                if r is not None and (best is None or r < best):
                    best, at = r, i
            if best is None:
                break
            sym[at:at + 2] = [sym[at] + sym[at + 1]]
        return [self.vocab[s] for s in sym if s in self.vocab]


@dataclass
class PromptCodes:  # prompt.rs:8
    num_codebooks: int
    cols: int
    data: np.ndarray  # [num_codebooks][cols] uint32, codebook-major


def load_prompt_codes(path) -> tuple[str, PromptCodes]:
    """prompt.rs:45-60: {"prompt_text", "num_codebooks", "cols", "codes"}."""
    try:
        doc = json.loads(Path(path).read_bytes())
    except (OSError, ValueError) as e:
        raise S2dError(-1, f"parse prompt codes json: {e}") from None
    codes = np.asarray(doc["codes"], dtype=np.uint32)
    expected = int(doc["cols"]) * int(doc["num_codebooks"])
    if codes.size != expected:
        raise S2dError(-1, f"prompt codes length mismatch: expected {expected} (cols={doc['cols']} * "
                           f"num_codebooks={doc['num_codebooks']}), got {codes.size}")
    return doc["prompt_text"], PromptCodes(int(doc["num_codebooks"]), int(doc["cols"]), codes)


def build_prompt(tokenizer: S2Tokenizer, text: str, num_codebooks: int, semantic_begin_id: int,
                 prompt_text: Optional[str] = None, prompt_codes: Optional[PromptCodes] = None) -> PromptTensor:
    """prompt.rs:105-220 build_prompt.  Without a reference (or with an
    empty reference text, no columns or another codebook count): the user
    turn and the assistant turn opening with <|voice|>.  With one: a system
    turn holding the reference text and, in place of its speech, the
    reference codes."""
    if (prompt_text is None) != (prompt_codes is None):
        raise S2dError(-1, "prompt_text and prompt_codes must both be set or both omitted")
    rows = num_codebooks + 1
    cfg = tokenizer.config
    nl = tokenizer.encode_newline()
    enc = tokenizer.encode_s2cpp
    post = (enc("<|im_start|>user") + nl + enc(text) + [cfg.im_end_id] + nl + enc("<|im_start|>assistant") + nl +
            [cfg.voice_id])
    has_ref = (prompt_codes is not None and prompt_text != "" and prompt_codes.cols > 0 and
               prompt_codes.num_codebooks == num_codebooks)
    if not has_ref:
        data = np.zeros((rows, len(post)), np.uint32)
        data[0] = post
        return PromptTensor(rows, len(post), data.reshape(-1))
    pre = (enc("<|im_start|>system") + nl +
           enc("convert the provided text to speech reference to the following:\n\nText:\n") +
           enc("<|speaker:0|>") + enc(prompt_text) + enc("\n\nSpeech:\n"))
    post = [cfg.im_end_id] + nl + post
    tp = prompt_codes.cols
    codes = np.asarray(prompt_codes.data, dtype=np.uint64).reshape(num_codebooks, tp)
    if int(codes[0].max(initial=0)) + semantic_begin_id > 0xFFFFFFFF:
        raise S2dError(-1, "prompt semantic id overflow")
    total = len(pre) + tp + len(post)
    data = np.zeros((rows, total), np.uint32)
    data[0, :len(pre)] = pre
    data[0, len(pre):len(pre) + tp] = codes[0] + semantic_begin_id
    data[1:, len(pre):len(pre) + tp] = codes
    data[0, len(pre) + tp:] = post
    return PromptTensor(rows, total, data.reshape(-1))
