"""The worker message host (engine/worker.js:139-200 restated in worker.py) driving the CUDA engine on a
GPU: load -> loaded, generate -> one token reply per id -> done, with the ids the oracle produces."""
import numpy as np
import pytest

from conftest import pkg
from oracle import oracle as O


@pytest.mark.gpu
def test_worker_load_generate_done_on_the_cuda_engine(cuda_ok):
    P = pkg()
    data = P.synthetic_pgw("tiny-llama", 3)
    posted = []
    w = P.DecodeWorker(posted.append)
    w.handle({"cmd": "load", "buffer": data, "modelId": "tiny"})
    assert posted[-1]["type"] == "loaded", posted[-1]
    assert posted[-1]["backend"] == "cuda" and posted[-1]["gpu"]["bytesAllocated"] > 0
    ids = [int(i) for i in P.seeded_prompt(20, 512, 41)]
    want = O.OracleModel(data).generate(ids, 12, eos=-1)["generatedIds"]
    n0 = len(posted)
    w.handle({"cmd": "generate", "promptIds": ids, "maxNewTokens": 12, "opts": {"ignoreEos": True}})
    replies = posted[n0:]
    assert [r["type"] for r in replies] == ["token"] * 12 + ["done"], [r.get("message") for r in replies]
    assert [r["id"] for r in replies[:12]] == want
    assert replies[0]["phase"] == "prefill" and all(r["phase"] == "decode" for r in replies[1:12])
    done = replies[-1]
    assert done["generatedIds"] == want and done["stopReason"] == "max_new_tokens"
    assert done["promptIds"] == ids and done["tokPerS"] > 0 and done["backend"] == "cuda"
    # speculation through the same message (opts.specK): same ids
    n1 = len(posted)
    w.handle({"cmd": "generate", "promptIds": ids, "maxNewTokens": 12, "opts": {"ignoreEos": True, "specK": 4}})
    assert posted[-1]["type"] == "done" and posted[-1]["generatedIds"] == want
    assert [r["id"] for r in posted[n1:-1]] == want
    w.handle({"cmd": "unload"})
    assert posted[-1]["type"] == "unloaded" and w.engine is None
