"""Byte-level BPE tokenizer and chat templates (engine/tokenizer.js) on the CPU.

The ids are pinned to HuggingFace `tokenizers` on the reference's tokenizer.json, through the reduced
spec and cases in tests/golden/tokenizer_cases.json (made by make_tokenizer_golden.py).  The chat
templates are checked against the rules of tokenizer.js:203-272.
"""
import importlib
import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
P = importlib.import_module("microllm-lab_b200")
T = importlib.import_module("microllm-lab_b200.tokenizer")
GOLDEN = os.path.join(ROOT, "tests", "golden", "tokenizer_cases.json")
S = T.SPECIAL


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN, encoding="utf-8") as f:
        return json.load(f)


@pytest.fixture(scope="module")
def tok(golden):
    return T.Tokenizer(golden["spec"])


def test_ids_match_huggingface_tokenizers(golden, tok):
    assert len(golden["cases"]) >= 16
    for case in golden["cases"]:
        assert tok.encode(case["text"]) == case["ids"], case["text"][:40]


def test_decode_round_trips(golden, tok):
    for case in golden["cases"]:
        assert tok.decode(case["ids"]) == case["text"]


def test_special_tokens_are_split_out_and_skippable(tok):
    ids = tok.encode("<|user|>hi<|assistant|>")
    assert ids[0] == S["USER"] and ids[-1] == S["ASSISTANT"] and len(ids) >= 3
    assert tok.decode(ids, skip_special=True) == "hi"
    assert tok.decode(ids) == "<|user|>hi<|assistant|>"
    assert tok.encode("") == [] and tok.encode(None) == []
    # an id outside the vocab decodes to nothing, as an undefined idToTok entry does
    assert tok.decode([10**6]) == ""


def test_invalid_utf8_is_replaced(tok):
    # the lone lead byte 0xC3 (first byte of "é", a case of the fixture) decodes to U+FFFD
    lead = tok.vocab[T._BYTE_TO_UNI[0xC3]]
    assert tok.decode([lead]) == "\ufffd"
    assert tok.decode([lead] + tok.encode("a")) == "\ufffda"


def test_petitgpt_template(tok):
    hi = tok.encode("hi")
    assert T.encode_messages(tok, [{"role": "user", "content": "hi"}], {}) == [S["BOS"], S["USER"], *hi, S["ASSISTANT"]]
    # default system turn, assistant turns closed by EOS, roles trimmed and lower-cased
    ids = T.encode_messages(tok, [{"role": " User ", "content": "hi"}, {"role": "assistant", "content": "a"},
                                  {"role": "user", "content": "hi"}], {"defaultSystem": "x"})
    assert ids == [S["BOS"], S["SYSTEM"], *tok.encode("x"), S["USER"], *hi, S["ASSISTANT"], *tok.encode("a"),
                   S["EOS"], S["USER"], *hi, S["ASSISTANT"]]
    # card ids replace the defaults
    card = {"bosId": 40, "eosId": 41, "specials": {"<|user|>": 42, "<|assistant|>": 43}}
    assert T.encode_messages(tok, [{"role": "user", "content": "hi"}], card) == [40, 42, *hi, 43]
    with pytest.raises(ValueError, match="invalid role"):
        T.encode_messages(tok, [{"role": "tool", "content": "hi"}], {})
    with pytest.raises(ValueError, match="empty message"):
        T.encode_messages(tok, [{"role": "user", "content": ""}], {})
    with pytest.raises(ValueError, match="end with a user turn"):
        T.encode_messages(tok, [{"role": "user", "content": "hi"}, {"role": "assistant", "content": "a"}], {})


def test_chatml_and_completion_templates(tok):
    nl = tok.encode("\n")
    card = {"template": "chatml", "bosId": 50, "eosId": 51, "defaultSystem": "s"}
    ids = T.encode_messages(tok, [{"role": "user", "content": "hi"}], card)
    want = [50, *tok.encode("system"), *nl, *tok.encode("s"), 51, *nl,
            50, *tok.encode("user"), *nl, *tok.encode("hi"), 51, *nl,
            50, *tok.encode("assistant"), *nl]
    assert ids == want
    # without card ids the chatml markers fall back to 1 and 2
    ids = T.encode_messages(tok, [{"role": "user", "content": "hi"}], {"template": "chatml"})
    assert ids[0] == 1 and ids.count(2) >= 1
    assert T.encode_messages(tok, [{"role": "user", "content": "a"}, {"role": "user", "content": "hi"}],
                             {"template": "completion"}) == tok.encode("hi")
    assert T.encode_messages(tok, [], {"template": "completion"}) == []


def test_worker_encodes_text_prompts_with_the_tokenizer(tok):
    class Eng:
        cfg = {"maxSeqLen": 256}
        bytesAllocated = 0
        calls = []

        def generate(self, ids, maxNewTokens, eosId, onToken, specK, ngram):
            self.calls.append(list(ids))
            out = tok.encode(" fox")
            for i, t in enumerate(out):
                onToken(t, {"phase": "prefill" if i == 0 else "decode"})
            return {"generatedIds": out, "stopReason": "max_new_tokens", "ttftMs": 0.1}

        def destroy(self):
            pass

    posted = []
    eng = Eng()
    w = P.DecodeWorker(posted.append, tokenizer=tok, engine_factory=lambda buf: eng)
    w.handle({"cmd": "load", "buffer": b"x"})
    w.handle({"cmd": "generate", "prompt": "The quick brown", "maxNewTokens": 8})
    assert eng.calls[-1] == [S["BOS"], S["USER"], *tok.encode("The quick brown"), S["ASSISTANT"]]
    assert posted[-1]["type"] == "done" and posted[-1]["text"] == " fox"
    assert "".join(m["piece"] for m in posted if m["type"] == "token") == " fox"


def test_worker_load_takes_a_tokenizer_spec(golden):
    class Eng:
        cfg = {"maxSeqLen": 256}
        bytesAllocated = 0

        def generate(self, ids, maxNewTokens, eosId, onToken, specK, ngram):
            self.ids = list(ids)
            return {"generatedIds": [], "stopReason": "max_new_tokens", "ttftMs": 0.0}

        def destroy(self):
            pass

    posted, eng = [], Eng()
    w = P.DecodeWorker(posted.append, engine_factory=lambda buf: eng)
    w.handle({"cmd": "load", "buffer": b"x", "tokenizerSpec": golden["spec"]})
    w.handle({"cmd": "generate", "prompt": "Hello, world!", "maxNewTokens": 4})
    hello = next(c["ids"] for c in golden["cases"] if c["text"] == "Hello, world!")
    assert eng.ids == [S["BOS"], S["USER"], *hello, S["ASSISTANT"]]
    assert posted[-1]["type"] == "done" and posted[-1]["text"] == ""
