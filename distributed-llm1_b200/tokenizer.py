"""Text in and out of the decode loop: the Qwen2 byte-level BPE tokenizer and the
chat template of the reference's chat box (script.js:175-200).

The reference loads `AutoTokenizer.from_pretrained("Qwen/Qwen2.5-1.5B-Instruct")`
from @huggingface/transformers over the network (script.js:176-179), encodes the
templated prompt without adding special tokens (script.js:198-199) and decodes
the generated ids with special tokens kept (script.js:186-190). This module reads
the same `tokenizer.json` a checkpoint ships and implements that pipeline:

  added tokens (<|im_start|>, <|im_end|>, ...) are cut out of the text first and
  map to their ids; every other piece is NFC-normalised, split by the
  pre-tokenizer's regex (taken from the file), mapped byte by byte to the
  byte-level alphabet (the GPT-2 byte -> printable-character table) and merged
  by BPE in merge-rank order; decoding maps the characters back to bytes and
  reads them as UTF-8.

No tokenizer file is in this repository (the checkpoint's is absent); the tests
use a small tokenizer in the same format built by tests/golden/make_tokenizer.py
and check every id against the `tokenizers` library on the same file.
"""
from __future__ import annotations

import json
import unicodedata

import regex

# The system prompt and turn markers of script.js:198.
SYSTEM_PROMPT = "You are a helpful assistant."


def chat_template(user_text: str, system: str = SYSTEM_PROMPT) -> str:
    """The prompt string of script.js:198 for one user turn."""
    return (f"<|im_start|>system\n{system}<|im_end|>\n"
            f"<|im_start|>user\n{user_text}<|im_end|>\n"
            f"<|im_start|>assistant\n")


def _byte_alphabet() -> dict[int, str]:
    """Byte -> character table of byte-level BPE: printable Latin-1 bytes map to
    themselves, the other 68 bytes to code points 256.. in byte order."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAC + 1)) + list(range(0xAE, 0xFF + 1))
    table, extra = {}, 0
    for b in range(256):
        if b in keep:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + extra)
            extra += 1
    return table


BYTE_TO_CHAR = _byte_alphabet()
CHAR_TO_BYTE = {c: b for b, c in BYTE_TO_CHAR.items()}


class Qwen2Tokenizer:
    """Byte-level BPE from a Hugging Face `tokenizer.json` (Qwen2 layout)."""

    def __init__(self, spec: dict):
        model = spec["model"]
        if model.get("type", "BPE") != "BPE":
            raise ValueError(f"unsupported tokenizer model {model.get('type')!r}")
        self.vocab: dict[str, int] = dict(model["vocab"])
        merges = model.get("merges", [])
        self.ranks: dict[tuple[str, str], int] = {}
        for i, m in enumerate(merges):
            a, b = (m.split(" ", 1) if isinstance(m, str) else m)
            self.ranks[(a, b)] = i
        self.ignore_merges = bool(model.get("ignore_merges", False))
        self.added = {t["content"]: t["id"] for t in spec.get("added_tokens", [])}
        self.special_ids = {t["id"] for t in spec.get("added_tokens", []) if t.get("special")}
        self.id_to_token = {i: t for t, i in self.vocab.items()}
        self.id_to_token.update({i: t for t, i in self.added.items()})
        self.nfc = self._has_nfc(spec.get("normalizer"))
        self.split = self._split_pattern(spec.get("pre_tokenizer"))
        # longest added token first, so overlapping markers resolve the long way
        alts = sorted(self.added, key=len, reverse=True)
        self.added_re = regex.compile("|".join(regex.escape(a) for a in alts)) if alts else None
        self._cache: dict[str, list[int]] = {}

    @classmethod
    def from_file(cls, path: str) -> "Qwen2Tokenizer":
        with open(path, encoding="utf-8") as f:
            return cls(json.load(f))

    @staticmethod
    def _has_nfc(norm) -> bool:
        if not norm:
            return False
        if norm.get("type") == "NFC":
            return True
        return any(n.get("type") == "NFC" for n in norm.get("normalizers", []))

    @staticmethod
    def _split_pattern(pre):
        pats = []

        def walk(p):
            if not p:
                return
            if p.get("type") == "Sequence":
                for q in p.get("pretokenizers", []):
                    walk(q)
            elif p.get("type") == "Split":
                pat = p["pattern"]
                pats.append(pat.get("Regex") or regex.escape(pat.get("String", "")))
        walk(pre)
        return regex.compile(pats[0]) if pats else None

    # ---- encoding ------------------------------------------------------------------
    def _bpe(self, word: str) -> list[int]:
        hit = self._cache.get(word)
        if hit is not None:
            return hit
        if self.ignore_merges and word in self.vocab:
            out = [self.vocab[word]]
        else:
            parts = list(word)
            while len(parts) > 1:
                best, at = None, -1
                for i in range(len(parts) - 1):
                    r = self.ranks.get((parts[i], parts[i + 1]))
                    if r is not None and (best is None or r < best):
                        best, at = r, i
                if best is None:
                    break
                parts[at:at + 2] = [parts[at] + parts[at + 1]]
            out = [self.vocab[p] for p in parts]
        self._cache[word] = out
        return out

    def _encode_plain(self, text: str) -> list[int]:
        if self.nfc:
            text = unicodedata.normalize("NFC", text)
        pieces = self.split.findall(text) if self.split else [text]
        ids = []
        for p in pieces:
            if p:
                ids += self._bpe("".join(BYTE_TO_CHAR[b] for b in p.encode("utf-8")))
        return ids

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        """Ids of `text`; added tokens in the text map to their ids. Qwen2 adds no
        BOS/EOS, so `add_special_tokens` changes nothing (script.js:199 passes false)."""
        ids, pos = [], 0
        if self.added_re is not None:
            for m in self.added_re.finditer(text):
                ids += self._encode_plain(text[pos:m.start()])
                ids.append(self.added[m.group(0)])
                pos = m.end()
        ids += self._encode_plain(text[pos:])
        return ids

    # ---- decoding ------------------------------------------------------------------
    def decode(self, ids, skip_special_tokens: bool = False) -> str:
        """Text of `ids` (script.js:188: special tokens kept by default)."""
        out, buf = [], bytearray()
        for i in ids:
            i = int(i)
            if i in self.special_ids and skip_special_tokens:
                continue
            tok = self.id_to_token.get(i)
            if tok is None:
                raise KeyError(f"token id {i} is not in the vocabulary")
            if i in self.added.values() and tok in self.added:
                out.append(buf.decode("utf-8", errors="replace"))
                buf = bytearray()
                out.append(tok)
            else:
                buf += bytes(CHAR_TO_BYTE[c] for c in tok)
        out.append(buf.decode("utf-8", errors="replace"))
        return "".join(out)

    def encode_chat(self, user_text: str, system: str = SYSTEM_PROMPT) -> list[int]:
        """Prompt ids of one chat turn (script.js:198-199)."""
        return self.encode(chat_template(user_text, system), add_special_tokens=False)
