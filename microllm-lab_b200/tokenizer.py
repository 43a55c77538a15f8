"""Byte-level BPE tokenizer and chat templates, restating the reference's engine/tokenizer.js.

This is host code for turning prompts into ids for the decode engine and ids back into text. It is not
on the device path. The rules follow the reference:
  - pre-tokenisation by the GPT-2 pattern with Unicode letter / number classes (tokenizer.js:3-4);
  - the GPT-2 byte-to-unicode table (tokenizer.js:6-28);
  - greedy lowest-rank pair merging (tokenizer.js:36-56);
  - special tokens split out of the text, longest first (tokenizer.js:89-124);
  - unknown pieces mapped to unk_token's id (default 1);
  - text cut to its last 32,768 characters;
  - decode through the reverse vocab, with special ids optionally skipped and invalid UTF-8 replaced
    (tokenizer.js:158-176);
  - the `petitgpt`, `chatml` and `completion` chat templates of `encodeMessages` (tokenizer.js:203-272).

One difference: lengths count code points, where JavaScript counts UTF-16 units. This only matters for
text above 32,768 characters that holds characters outside the BMP.
"""
from __future__ import annotations

import json

import regex

# tokenizer.js:3-4 (the `u` flag's \p classes; `regex` supports them)
_PAT = regex.compile(r"""'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+""")
_MAX_CHARS = 32768
SPECIAL = {"PAD": 0, "UNK": 1, "BOS": 2, "EOS": 3, "SYSTEM": 4, "USER": 5, "ASSISTANT": 6}  # tokenizer.js:188-196


def _bytes_to_unicode():
    """GPT-2's reversible byte <-> printable character table."""
    bs = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    cs = bs[:]
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    return {b: chr(c) for b, c in zip(bs, cs)}


_BYTE_TO_UNI = _bytes_to_unicode()
_UNI_TO_BYTE = {c: b for b, c in _BYTE_TO_UNI.items()}


def _bpe(word: str, ranks: dict) -> list:
    """Merge the lowest-ranked adjacent pair until none is in the merge table (first pair on ties)."""
    parts = list(word)
    while len(parts) > 1:
        best, best_i = None, -1
        for i in range(len(parts) - 1):
            r = ranks.get((parts[i], parts[i + 1]))
            if r is not None and (best is None or r < best):
                best, best_i = r, i
        if best_i < 0:
            break
        parts[best_i:best_i + 2] = [parts[best_i] + parts[best_i + 1]]
    return parts


class Tokenizer:
    def __init__(self, spec: dict):
        model = spec["model"]
        self.vocab = dict(model["vocab"])
        unk = self.vocab.get(model.get("unk_token"))
        self.unk_id = 1 if unk is None else unk
        self.ranks = {}
        for i, m in enumerate(model.get("merges") or []):
            if isinstance(m, str):
                a, _, b = m.partition(" ")
            else:
                a, b = m[0], m[1]
            self.ranks[(a, b)] = i  # a repeated pair keeps its last rank, as Map.set does
        self.special = {t["content"]: t["id"] for t in spec.get("added_tokens") or [] if t.get("special")}
        self._special_list = sorted(self.special, key=len, reverse=True)
        self._special_ids = set(self.special.values())
        self._id_to_tok = {i: t for t, i in self.vocab.items()}
        self.vocab_size = len(self.vocab)

    @classmethod
    def from_file(cls, path: str) -> "Tokenizer":
        with open(path, encoding="utf-8") as f:
            return cls(json.load(f))

    def _encode_raw(self, text: str) -> list:
        ids = []
        for part in _PAT.findall(text) or ([text] if text else []):
            mapped = "".join(_BYTE_TO_UNI[b] for b in part.encode("utf-8"))
            for piece in _bpe(mapped, self.ranks):
                ids.append(self.vocab.get(piece, self.unk_id))
        return ids

    def encode(self, text) -> list:
        if not text:
            return []
        text = str(text)
        if len(text) > _MAX_CHARS:
            text = text[len(text) - _MAX_CHARS:]
        if not self._special_list:
            return self._encode_raw(text)
        ids, i, n = [], 0, len(text)
        while i < n:
            hit = next((s for s in self._special_list if text.startswith(s, i)), None)
            if hit is not None:
                ids.append(self.special[hit])
                i += len(hit)
                continue
            j = i + 1
            while j <= n and not any(text.startswith(s, j) for s in self._special_list):
                j += 1
            ids.extend(self._encode_raw(text[i:j]))
            i = j
        return ids

    def decode(self, ids, skip_special: bool = False) -> str:
        mapped = []
        for i in ids:
            i = int(i)
            if skip_special and i in self._special_ids:
                continue
            piece = self._id_to_tok.get(i)
            if piece:
                mapped.append(piece)
        data = bytes(_UNI_TO_BYTE[c] for c in "".join(mapped) if c in _UNI_TO_BYTE)
        return data.decode("utf-8", errors="replace")

    def encode_messages(self, messages, card=None) -> list:
        return encode_messages(self, messages, card or {})


def encode_messages(tok: Tokenizer, messages, card: dict) -> list:
    """Chat template of a model card (tokenizer.js:203-272): `petitgpt` (default), `chatml`, `completion`."""
    msgs = []
    for m in messages:
        content = m.get("content")
        content = "" if content is None else str(content)
        if len(content) > _MAX_CHARS:
            content = content[len(content) - _MAX_CHARS:]
        msgs.append({"role": str(m.get("role")).strip().lower(), "content": content})
    specials = card.get("specials") or {}

    def pick(*vals):  # JavaScript `a ?? b ?? ...`
        return next((v for v in vals if v is not None), None)

    tpl = card.get("template") or "petitgpt"
    if tpl == "completion":
        return tok.encode(msgs[-1]["content"] if msgs else "")
    if tpl == "chatml":
        sys_msg = card.get("defaultSystem")
        if sys_msg and (not msgs or msgs[0]["role"] != "system"):
            msgs.insert(0, {"role": "system", "content": sys_msg})
        im_start = pick(tok.special.get("<|im_start|>"), specials.get("<|im_start|>"), card.get("bosId"), 1)
        im_end = pick(tok.special.get("<|im_end|>"), specials.get("<|im_end|>"), card.get("eosId"), 2)
        ids = []
        for m in msgs:
            ids += [im_start] + tok.encode(m["role"]) + tok.encode("\n") + tok.encode(m["content"])
            ids += [im_end] + tok.encode("\n")
        return ids + [im_start] + tok.encode("assistant") + tok.encode("\n")
    default_system = card.get("defaultSystem") or None
    if default_system and (not msgs or msgs[0]["role"] != "system"):
        msgs.insert(0, {"role": "system", "content": default_system})
    bos = pick(card.get("bosId"), SPECIAL["BOS"])
    eos = pick(card.get("eosId"), SPECIAL["EOS"])
    role_id = {
        "system": pick(specials.get("<|system|>"), SPECIAL["SYSTEM"]),
        "user": pick(specials.get("<|user|>"), SPECIAL["USER"]),
        "assistant": pick(specials.get("<|assistant|>"), SPECIAL["ASSISTANT"]),
    }
    ids = [bos]
    for m in msgs:
        if role_id.get(m["role"]) is None:
            raise ValueError(f"invalid role {m['role']}")
        content_ids = tok.encode(m["content"])
        if not content_ids:
            raise ValueError("empty message encoding")
        ids.append(role_id[m["role"]])
        ids += content_ids
        if m["role"] == "assistant":
            ids.append(eos)
    if not msgs or msgs[-1]["role"] != "user":
        raise ValueError("prompt must end with a user turn")
    ids.append(role_id["assistant"])
    return ids
