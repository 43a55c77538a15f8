"""GPU token streaming (mllm_generate_stream, the onToken path of engine/infer.js:615,630 and
engine/webgpu.js:1202-1237,1253,1265): ids reach onToken in order, equal to the oracle's, while the
device is still generating."""
import time

import pytest

from conftest import pkg
from oracle import oracle as O


def _run(eng, ids, n, **kw):
    got = []
    t0 = time.perf_counter()
    res = eng.generate(ids, maxNewTokens=n, eosId=-1,
                       onToken=lambda tok, meta: got.append((time.perf_counter(), tok, meta)), **kw)
    return res, got, t0, time.perf_counter()


@pytest.mark.gpu
def test_stream_ids_in_order_equal_oracle(cuda_ok):
    P = pkg()
    data = P.synthetic_pgw("tiny-llama", 3)
    eng = P.CudaPetitGPT(data)
    try:
        om = O.OracleModel(data)
        ids = P.seeded_prompt(14, 512, 71)
        want = om.generate(ids, 40, eos=-1)["generatedIds"]
        res, got, _, _ = _run(eng, ids, 40)
        assert [g[1] for g in got] == want == res["generatedIds"]
        assert got[0][2]["phase"] == "prefill" and "ms" in got[0][2]
        assert all(g[2]["phase"] == "decode" for g in got[1:])
        # speculation: the verify loop streams r0 as "decode" and accepted drafts as "spec"
        span = P.copy_span_prompt(96, 512, 72)
        ref = om.generate_spec(span, 40, eos=-1, spec_k=4, ngram=3)
        res, got, _, _ = _run(eng, span, 40, specK=4, ngram=3)
        assert [g[1] for g in got] == ref["generatedIds"] == res["generatedIds"]
        assert sum(g[2]["phase"] == "spec" for g in got) == ref["specHits"] == res["specHits"]
    finally:
        eng.destroy()


@pytest.mark.gpu
def test_stream_first_id_arrives_before_the_launch_ends(cuda_ok):
    """PetitGPT shape, 64-token prompt, 128 ids: the first id reaches the host while the decode loop
    (one persistent launch) still has most of its 127 steps to run, and the ids arrive spread over it."""
    P = pkg()
    data = P.synthetic_pgw("petitgpt", 0, cache_dir="/tmp/mllm_pgw_cache")
    eng = P.CudaPetitGPT(data)
    try:
        ids = P.seeded_prompt(64, 32000, 0)
        plain = eng.generate(ids, maxNewTokens=128, eosId=-1)["generatedIds"]
        res, got, t0, t1 = _run(eng, ids, 128)
        assert [g[1] for g in got] == plain == res["generatedIds"]
        span = t1 - t0
        assert got[0][0] - t0 < 0.25 * span, (got[0][0] - t0, span)
        assert got[63][0] - t0 < 0.85 * span, (got[63][0] - t0, span)
    finally:
        eng.destroy()
