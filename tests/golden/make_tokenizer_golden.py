#!/usr/bin/env python3
"""Regenerate tests/golden/tokenizer_cases.json from the reference's tokenizer.json.

Run where the reference project is mounted, with MLLM_REFERENCE_DIR set to its root. It needs the
HuggingFace `tokenizers` package. The reference's engine/tokenizer.js:1 states that its byte-level BPE
matches HuggingFace tokenizers on this file, so HF's ids are the pin.

The fixture holds:
  - "cases": fixed strings and the ids HF `tokenizers` gives for them with the full tokenizer.json
    (no added BOS/EOS);
  - "spec": a reduced tokenizer.json. It keeps the vocab entries and merges whose strings occur inside
    the byte-level pieces of those strings, with the merges in their original order, plus every special
    token. A BPE merge can only fire on a piece that contains its result, so the reduced spec encodes
    the cases exactly as the full one does.

The tests then need neither the 2.2 MB file nor `tokenizers`.

Before writing, the script checks the product tokenizer (microllm-lab_b200/tokenizer.py) against HF on
the full file, over 3,000 seeded random strings. The strings mix scripts, emoji, digits, punctuation,
contractions, whitespace runs and special-token text. The script stops on the first difference.
"""
import importlib
import json
import os
import random
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("MLLM_REFERENCE_DIR", "")

CASES = [
    "Hello, world!",
    "  leading spaces and  double  spaces  ",
    "numbers 12345 and 3.14159",
    "it's we're they've I'm you'll he'd",
    "Ünïcödé — naïve café ☕ 日本語 テキスト",
    "tabs\tand\nnewlines\n\n",
    "emoji 🎉🚀 end",
    "<|user|>hi<|assistant|>",
    "[BOS]x[EOS]",
    "",
    "a",
    "   ",
    "mixed123abc!!!???",
    "UPPER lower MiXeD",
    " nbsp emspace",
    "x" * 300,
    "The quick brown fox jumps over the lazy dog.",
    "user\n",
    "assistant",
    "Once upon a time, there was a little robot named Petit.",
]


def stress_check(path, hf, n=3000, seed=7):
    """Product tokenizer vs HF on seeded random strings over the full tokenizer.json."""
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    T = importlib.import_module("microllm-lab_b200.tokenizer")
    tok = T.Tokenizer.from_file(path)
    rng = random.Random(seed)
    alph = (list("abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789 .,;:!?'\"-_()[]{}<>|/\\@#$%^&*+=~`\t\n")
            + list("éèüößçñØåÆœ€£¥—–…“”‘’") + list("日本語中文한국어テキストабвгдеёжзиαβγδεζ")
            + ["🎉", "🚀", "👍🏽", "\u00a0", "\u2003", "\u200b"])
    specials = ["<|user|>", "<|assistant|>", "<|system|>", "[BOS]", "[EOS]", "[PAD]", "[UNK]"]
    for _ in range(n):
        parts = []
        for _ in range(rng.randint(0, 60)):
            r = rng.random()
            if r < 0.03:
                parts.append(rng.choice(specials))
            elif r < 0.08:
                parts.append("'" + rng.choice(["s", "t", "re", "ve", "m", "ll", "d"]))
            elif r < 0.15:
                parts.append(" " * rng.randint(1, 4))
            else:
                parts.append(rng.choice(alph))
        text = "".join(parts)
        want = hf.encode(text, add_special_tokens=False).ids
        got = tok.encode(text)
        if got != want:
            raise SystemExit(f"tokenizer differs from HF on {text!r}: {got[:12]} vs {want[:12]}")
        if tok.decode(got) != hf.decode(want, skip_special_tokens=False):
            raise SystemExit(f"decode differs from HF on {text!r}")
    print(f"product tokenizer = HF on {n} random strings")


def main():
    if not REF or not os.path.isdir(REF):
        raise SystemExit("set MLLM_REFERENCE_DIR to the reference project's root directory")
    from tokenizers import Tokenizer
    path = os.path.join(REF, "tokenizer.json")
    with open(path, encoding="utf-8") as f:
        spec = json.load(f)
    hf = Tokenizer.from_file(path)
    stress_check(path, hf)
    specials = [t["content"] for t in spec.get("added_tokens", []) if t.get("special")]
    split = re.compile("|".join(re.escape(s) for s in sorted(specials, key=len, reverse=True)))
    pieces = set()
    for text in CASES:
        for seg in split.split(text):
            if seg:
                pieces.update(p for p, _ in hf.pre_tokenizer.pre_tokenize_str(seg))
    subs = set()
    for p in pieces:
        for i in range(len(p)):
            for j in range(i + 1, len(p) + 1):
                subs.add(p[i:j])
    model = spec["model"]
    keep_tokens = subs | set(specials) | {model.get("unk_token")}
    vocab = {t: i for t, i in model["vocab"].items() if t in keep_tokens}
    merges = []
    for m in model["merges"]:
        a, b = (m.split(" ", 1) if isinstance(m, str) else m)
        if a + b in subs:
            merges.append([a, b])
    reduced = {
        "model": {"type": "BPE", "unk_token": model.get("unk_token"), "vocab": vocab, "merges": merges},
        "added_tokens": [t for t in spec.get("added_tokens", []) if t.get("special")],
    }
    out = {
        "source": "tokenizer.json of the reference project, encoded with HuggingFace tokenizers "
                  "(add_special_tokens=False)",
        "spec": reduced,
        "cases": [{"text": t, "ids": hf.encode(t, add_special_tokens=False).ids} for t in CASES],
    }
    dst = os.path.join(HERE, "tokenizer_cases.json")
    with open(dst, "w", encoding="utf-8") as f:
        json.dump(out, f, ensure_ascii=False, separators=(",", ":"))
    print(dst, os.path.getsize(dst), "bytes;", len(vocab), "vocab entries,", len(merges), "merges")


if __name__ == "__main__":
    main()
