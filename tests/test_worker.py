"""The worker message host (engine/worker.js:16-200) on the CPU, driven with a fake engine and tokenizer.

The fake engine has the surface of ``CudaPetitGPT`` that the host uses (``cfg``, ``bytesAllocated``,
``generate``, ``destroy``) and records its calls, so that the protocol rules can be checked without a
device:
  - replies and their fields;
  - prompt truncation with a kept BOS;
  - the EOS choice;
  - per-token replies;
  - error replies;
  - engine lifetime.
"""
import importlib
import importlib.util
import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
P = importlib.import_module("microllm-lab_b200")
BOS, EOS = P.SPECIAL["BOS"], P.SPECIAL["EOS"]


class FakeEngine:
    def __init__(self, buffer, out=(11, 12, 13), max_seq=32):
        self.buffer = buffer
        self.cfg = {"arch": "llama", "vocabSize": 64, "maxSeqLen": max_seq}
        self.bytesAllocated = 1234
        self.out = list(out)
        self.calls = []
        self.destroyed = False

    def generate(self, ids, maxNewTokens=64, eosId=EOS, onToken=None, specK=0, ngram=3):
        self.calls.append(dict(ids=list(ids), maxNewTokens=maxNewTokens, eosId=eosId, specK=specK, ngram=ngram))
        gen = self.out[:maxNewTokens]
        if onToken:
            for i, t in enumerate(gen):
                onToken(t, {"phase": "prefill" if i == 0 else "decode"})
        stop = "eos" if gen and gen[-1] == eosId else "max_new_tokens"
        return {"generatedIds": gen, "stopReason": stop, "ttftMs": 1.5, "totalMs": 3.0}

    def destroy(self):
        self.destroyed = True


class FakeTokenizer:
    """Chat template = [BOS, USER, one id per character (100 + ord % 50)]; decode = ids joined."""

    def encode_messages(self, messages, card):
        text = messages[-1]["content"]
        return [BOS, P.SPECIAL["USER"]] + [100 + ord(c) % 50 for c in text]

    def decode(self, ids, skip_special=False):
        ids = [i for i in ids if not (skip_special and i < 7)]
        return " ".join(str(i) for i in ids)


def make(out=(11, 12, 13), max_seq=32, tokenizer=None):
    posted, engines = [], []

    def factory(buf):
        engines.append(FakeEngine(buf, out, max_seq))
        return engines[-1]

    return P.DecodeWorker(posted.append, tokenizer=tokenizer, engine_factory=factory), posted, engines


def test_ping_and_unknown_commands():
    w, posted, _ = make()
    w.handle({"cmd": "ping"})
    w.handle({"cmd": "no-such-command"})
    w.handle(None)
    assert posted == [{"type": "pong"}]


def test_generate_before_load_is_an_error_reply():
    w, posted, _ = make()
    w.handle({"cmd": "generate", "promptIds": [1, 2]})
    assert posted[-1]["type"] == "error" and posted[-1]["message"] == "no model loaded"
    assert "stack" in posted[-1]


def test_load_reply_and_model_id_rule():
    w, posted, engines = make()
    w.handle({"cmd": "load", "buffer": b"pgw", "kind": "q4"})
    m = posted[-1]
    assert m["type"] == "loaded" and m["modelId"] == "q4" and m["dtype"] == "q4" and m["backend"] == "cuda"
    assert m["gpu"]["bytesAllocated"] == 1234 and m["cfg"]["maxSeqLen"] == 32
    assert engines[0].buffer == b"pgw"
    w.handle({"cmd": "load", "buffer": b"pgw2"})
    assert posted[-1]["modelId"] == "petitgpt"
    # a new load destroys the previous engine first
    assert engines[0].destroyed and not engines[1].destroyed
    w.handle({"cmd": "unload"})
    assert posted[-1] == {"type": "unloaded"} and engines[1].destroyed and w.engine is None
    w.handle({"cmd": "load"})
    assert posted[-1]["type"] == "error"


def test_generate_tokens_done_and_eos_rules():
    tok = FakeTokenizer()
    w, posted, engines = make(out=(21, 22, EOS), tokenizer=tok)
    w.handle({"cmd": "load", "buffer": b"x", "card": {"maxSeqLen": 128}})
    posted.clear()
    w.handle({"cmd": "generate", "prompt": "hi", "maxNewTokens": 0})  # `|| 64`
    call = engines[0].calls[-1]
    assert call["maxNewTokens"] == 64 and call["eosId"] == EOS and call["specK"] == 0
    assert call["ids"] == [BOS, P.SPECIAL["USER"], 100 + ord("h") % 50, 100 + ord("i") % 50]
    assert [m["type"] for m in posted] == ["token", "token", "token", "done"]
    assert [m["id"] for m in posted[:3]] == [21, 22, EOS]
    assert [m["phase"] for m in posted[:3]] == ["prefill", "decode", "decode"]
    assert posted[0]["piece"] == "21"
    done = posted[-1]
    assert done["generatedIds"] == [21, 22, EOS] and done["stopReason"] == "eos"
    assert done["text"] == "21 22"  # final EOS dropped, specials skipped
    assert done["raw"] == "21 22 3"
    assert done["promptIds"] == call["ids"] and done["ttftMs"] == 1.5
    assert done["tokPerS"] == pytest.approx(3 / (done["totalMs"] / 1000))
    # ignoreEos: eosId -1, nothing is stripped; the card's eosId wins otherwise
    w.handle({"cmd": "generate", "prompt": "hi", "maxNewTokens": 3, "opts": {"ignoreEos": True, "specK": 4}})
    assert engines[0].calls[-1]["eosId"] == -1 and engines[0].calls[-1]["specK"] == 4
    assert posted[-1]["text"] == "21 22"  # the EOS id is still a special id for the text
    w.handle({"cmd": "load", "buffer": b"x", "card": {"eosId": 22, "maxSeqLen": 64}})
    w.handle({"cmd": "generate", "prompt": "hi", "maxNewTokens": 3})
    assert engines[1].calls[-1]["eosId"] == 22


def test_prompt_truncation_keeps_bos():
    w, posted, engines = make(max_seq=16)
    w.handle({"cmd": "load", "buffer": b"x"})
    ids = [BOS] + list(range(100, 120))
    # maxPrompt = max(1, 16 - 8 - 4) = 4: BOS + the last 3 ids
    w.handle({"cmd": "generate", "promptIds": ids, "maxNewTokens": 8})
    assert engines[0].calls[-1]["ids"] == [BOS, 117, 118, 119]
    # without a leading BOS: the last 4 ids
    w.handle({"cmd": "generate", "promptIds": ids[1:], "maxNewTokens": 8})
    assert engines[0].calls[-1]["ids"] == [116, 117, 118, 119]
    # a numeric string counts as its number
    w.handle({"cmd": "generate", "promptIds": ids, "maxNewTokens": "8"})
    assert engines[0].calls[-1]["ids"] == [BOS, 117, 118, 119] and engines[0].calls[-1]["maxNewTokens"] == 8
    # maxPrompt floors at 1: BOS alone survives
    w.handle({"cmd": "generate", "promptIds": ids, "maxNewTokens": 30})
    assert engines[0].calls[-1]["ids"] == [BOS]
    # a card bosId replaces the default; an explicit None falls back to it (JS `??`)
    w.handle({"cmd": "load", "buffer": b"x", "card": {"bosId": 100, "maxSeqLen": 16}})
    w.handle({"cmd": "generate", "promptIds": ids[1:], "maxNewTokens": 8})
    assert engines[1].calls[-1]["ids"] == [100, 117, 118, 119]
    w.handle({"cmd": "load", "buffer": b"x", "card": {"bosId": None, "maxSeqLen": 16}})
    w.handle({"cmd": "generate", "promptIds": ids, "maxNewTokens": 8})
    assert engines[2].calls[-1]["ids"] == [BOS, 117, 118, 119]
    # text fields are None without a tokenizer; a text prompt needs one
    assert posted[-1]["type"] == "done" and posted[-1]["text"] is None
    w.handle({"cmd": "generate", "prompt": "hello"})
    assert posted[-1]["type"] == "error" and "promptIds" in posted[-1]["message"]


def test_fractional_max_new_and_js_truthiness():
    """engine/infer.js:625 loops `for (i = 1; i < maxNewTokens; i++)`: a fractional 3.5 (or "3.5") yields
    ceil(3.5) = 4 ids; maxPrompt = max(1, 16 - 3.5 - 4) = 8.5 keeps BOS + the ids from slice(trunc(21 -
    7.5)) = slice(13).  An empty tokenizerSpec object is truthy in JavaScript (it reaches the tokenizer
    loader, which rejects it); an empty string is not (the loaded tokenizer stays)."""
    w, posted, engines = make(max_seq=16)
    w.handle({"cmd": "load", "buffer": b"x"})
    ids = [BOS] + list(range(100, 120))
    for mx in (3.5, "3.5"):
        w.handle({"cmd": "generate", "promptIds": ids, "maxNewTokens": mx})
        call = engines[0].calls[-1]
        assert call["maxNewTokens"] == 4, mx
        assert call["ids"] == [BOS] + ids[13:], mx
    w.handle({"cmd": "generate", "promptIds": ids, "maxNewTokens": 8.7})
    assert engines[0].calls[-1]["maxNewTokens"] == 9
    tok = FakeTokenizer()
    w.handle({"cmd": "load", "buffer": b"x", "tokenizer": tok})
    w.handle({"cmd": "load", "buffer": b"x", "tokenizerSpec": ""})
    assert posted[-1]["type"] == "loaded" and w.tokenizer is tok
    w.handle({"cmd": "load", "buffer": b"x", "tokenizerSpec": {}})
    assert posted[-1]["type"] == "error"


@pytest.mark.skipif(importlib.util.find_spec("torch") is None, reason="torch absent")
def test_default_engine_without_a_device_is_an_error_reply():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present: the default engine would load")
    posted = []
    w = P.DecodeWorker(posted.append)
    data = P.synthetic_pgw("tiny-llama", 1, cache_dir="/tmp/mllm_pgw_cache")
    w.handle({"cmd": "load", "buffer": data})
    assert posted[-1]["type"] == "error" and w.engine is None and w.backend == "none"
