"""Layer-wise (token-batch) engine on the tensor cores, through the C ABI, against the CPU oracle:
multi-token forwards (prefill, verify rows) and the replicated multi-sequence decode
(mllm_generate_batch).

Bars: token ids and stop reasons bit-exact per sequence; logits max-abs <= 2e-2."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, pkg
from oracle import oracle as O

LOGIT_TOL = 2e-2


def _data(name):
    P = pkg()
    if name == "tiny-llama":
        return P.synthetic_pgw("tiny-llama", 3)
    if name == "tiny-gpt2":
        return P.synthetic_pgw("tiny-gpt2", 4)
    return open(os.path.join(GOLDEN, name.replace("-", "_") + ".pgw"), "rb").read()


def _engine(data, monkeypatch=None, env=None, **kw):
    """Engine created with extra environment knobs (read by mllm_create only)."""
    P = pkg()
    env = env or {}
    old = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        return P.CudaPetitGPT(data, **kw)
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


@pytest.fixture(scope="module")
def batch_models(cuda_ok):
    out = {}
    for name in ["tiny-llama", "tiny-gpt2", "ref-llama", "ref-gpt2"]:
        data = _data(name)
        out[name] = (data, _engine(data, max_slots=8), O.OracleModel(data))
    yield out
    for _, eng, _ in out.values():
        eng.destroy()


def _prompts(V, lens, seed):
    P = pkg()
    return [P.seeded_prompt(n, V, seed + i) for i, n in enumerate(lens)]


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["tiny-llama", "tiny-gpt2", "ref-llama", "ref-gpt2"])
def test_batch_matches_per_sequence_oracle(batch_models, name):
    """Each sequence of the batch equals engine/infer.js:603-646 run alone (GPT-2: argmaxGpt2 over
    that sequence's own ids)."""
    data, eng, om = batch_models[name]
    V = eng.cfg["vocabSize"]
    seqs = _prompts(V, [1, 5, 17, 33, 9, 12], 40)
    res, st = eng.generateBatch(seqs, maxNewTokens=32, eosId=-1)
    assert st["nSeq"] == len(seqs) and st["totalGenerated"] == 32 * len(seqs)
    for q, r in zip(seqs, res):
        ref = om.generate(q, 32, eos=-1)
        assert r["generatedIds"] == ref["generatedIds"]
        assert r["stopReason"] == ref["stopReason"]


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["tiny-llama", "ref-llama"])
def test_batch_wide_lm_head(cuda_ok, name):
    """96 sequences (>= 64 lm rows, no logits) take the lm_head on the tcgen05 tile: one 128-token tile
    holding 96 rows (12 blocks of 8); ref-llama's 96-id vocab also ends in a partial row tile.  Every
    sequence equals the oracle, the persistent mma.sync GEMM (MLLM_LWE_LM_TC5=0; two token tiles, the
    second partial) and the per-tile GEMM (both off)."""
    data = _data(name)
    om = O.OracleModel(data)
    engs = [_engine(data, max_slots=96),
            _engine(data, env={"MLLM_LWE_LM_TC5": "0"}, max_slots=96),
            _engine(data, env={"MLLM_LWE_LM_TC5": "0", "MLLM_LWE_LM_WIDE": "0"}, max_slots=96)]
    try:
        V = engs[0].cfg["vocabSize"]
        seqs = _prompts(V, [1 + (7 * i) % 23 for i in range(96)], 300)
        runs = [e.generateBatch(seqs, maxNewTokens=12, eosId=-1) for e in engs]
        assert runs[0][1]["nSeq"] == 96
        for i, q in enumerate(seqs):
            ids = [r[0][i]["generatedIds"] for r in runs]
            assert ids[0] == ids[1] == ids[2], i
            if i % 8 == 0:  # the oracle on every eighth sequence
                assert ids[0] == om.generate(q, 12, eos=-1)["generatedIds"], i
    finally:
        for e in engs:
            e.destroy()


@pytest.mark.gpu
def test_batch_wide_w13_prefill(cuda_ok):
    """A 640-row prefill chunk (8 prompts of 80 ids) takes the persistent w1/w3 GEMM: every sequence
    equals the oracle, and the engine without it (MLLM_LWE_W13_WIDE=0)."""
    data = _data("tiny-llama")
    om = O.OracleModel(data)
    eng = _engine(data, max_slots=8)
    ref_eng = _engine(data, env={"MLLM_LWE_W13_WIDE": "0"}, max_slots=8)
    try:
        V = eng.cfg["vocabSize"]
        seqs = _prompts(V, [80] * 8, 500)
        res, st = eng.generateBatch(seqs, maxNewTokens=10, eosId=-1)
        res0, _ = ref_eng.generateBatch(seqs, maxNewTokens=10, eosId=-1)
        assert st["prefillForwards"] == 1
        for i, (q, r, r0) in enumerate(zip(seqs, res, res0)):
            assert r["generatedIds"] == r0["generatedIds"], i
            assert r["generatedIds"] == om.generate(q, 10, eos=-1)["generatedIds"], i
    finally:
        eng.destroy()
        ref_eng.destroy()


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["tiny-llama", "ref-llama"])
def test_layer_gemms_on_tcgen05(cuda_ok, name):
    """MLLM_LWE_GEMM_TC5=1: forwards of >= 32 rows run every layer GEMM (QKV, proj + residual, w1/w3 +
    SiLU, w2 + residual) on the tcgen05 tile with the tiled activation layout.  A 100-token prompt's
    logits of every row within the logits bar of the oracle; 48 sequences (batched prefill and 48-row
    decode steps) equal the mma.sync engine's streams and the oracle's."""
    data = _data(name)
    om = O.OracleModel(data)
    eng = _engine(data, env={"MLLM_LWE_GEMM_TC5": "1"}, max_slots=48)
    ref_eng = _engine(data, max_slots=48)
    try:
        V = eng.cfg["vocabSize"]
        ids = pkg().seeded_prompt(100, V, 41)
        eng.resetCache()
        g, _ = eng.forward(ids, 0, logits_each=True)
        r = np.asarray(om.forward(ids, 0, logits_each=True))
        err = float(np.abs(g - r).max())
        assert err <= LOGIT_TOL, err
        seqs = _prompts(V, [1 + (5 * i) % 37 for i in range(48)], 700)
        res, st = eng.generateBatch(seqs, maxNewTokens=10, eosId=-1)
        res0, _ = ref_eng.generateBatch(seqs, maxNewTokens=10, eosId=-1)
        for i, (q, a, b) in enumerate(zip(seqs, res, res0)):
            assert a["generatedIds"] == b["generatedIds"], i
            if i % 6 == 0:
                assert a["generatedIds"] == om.generate(q, 10, eos=-1)["generatedIds"], i
    finally:
        eng.destroy()
        ref_eng.destroy()


@pytest.mark.gpu
def test_batch_single_sequence_equals_generate(batch_models):
    data, eng, om = batch_models["ref-llama"]
    ids = pkg().seeded_prompt(20, eng.cfg["vocabSize"], 50)
    res, _ = eng.generateBatch([ids], maxNewTokens=24, eosId=-1)
    assert res[0]["generatedIds"] == eng.generate(ids, maxNewTokens=24, eosId=-1)["generatedIds"]


@pytest.mark.gpu
def test_batch_stop_rules(batch_models):
    """EOS per sequence (the others keep going), maxNewTokens = 1, and the cache-length stop."""
    data, eng, om = batch_models["tiny-llama"]
    seqs = _prompts(512, [12, 7, 20, 3], 60)
    full = om.generate(seqs[0], 20, eos=-1)["generatedIds"]
    eos = full[5]
    res, _ = eng.generateBatch(seqs, maxNewTokens=20, eosId=eos)
    for q, r in zip(seqs, res):
        ref = om.generate(q, 20, eos=eos)
        assert r["generatedIds"] == ref["generatedIds"] and r["stopReason"] == ref["stopReason"]
    assert res[0]["stopReason"] == "eos" and len(res[0]["generatedIds"]) == 6
    res, st = eng.generateBatch(seqs, maxNewTokens=1, eosId=-1)
    assert [r["generatedIds"] for r in res] == [om.generate(q, 1, eos=-1)["generatedIds"] for q in seqs]
    assert st["steps"] == 0
    # maxNewTokens 170 > maxSeqLen 160: prompts cut to 1 id, decode stops at the cache length
    res, _ = eng.generateBatch(seqs[:3], maxNewTokens=170, eosId=-1)
    for q, r in zip(seqs[:3], res):
        ref = om.generate(q, 170, eos=-1)
        assert r["generatedIds"] == ref["generatedIds"]
        assert len(r["generatedIds"]) == 159


@pytest.mark.gpu
@pytest.mark.parametrize("env", [{"MLLM_LWE_TOKENS": "16"}, {"MLLM_LWE_GRAPH": "0"}])
def test_batch_chunked_prefill_and_plain_launches(cuda_ok, env):
    """16 token rows per forward (prompts split across forwards and forwards mixing sequences), and
    the decode step launched without a CUDA graph."""
    data = _data("tiny-llama")
    eng = _engine(data, env=env, max_slots=5)
    om = O.OracleModel(data)
    seqs = _prompts(512, [40, 3, 16, 17, 9], 70)
    res, st = eng.generateBatch(seqs, maxNewTokens=16, eosId=-1)
    if "MLLM_LWE_TOKENS" in env:
        assert st["prefillForwards"] == (sum(len(q) for q in seqs) + 15) // 16
    for q, r in zip(seqs, res):
        assert r["generatedIds"] == om.generate(q, 16, eos=-1)["generatedIds"]
    eng.destroy()


@pytest.mark.gpu
def test_batch_argument_errors(batch_models):
    P = pkg()
    data, eng, om = batch_models["tiny-llama"]
    with pytest.raises(P.MllmError, match="n_seq"):
        eng.generateBatch([[1, 2]] * 9, maxNewTokens=4)
    with pytest.raises(P.MllmError, match="empty prompt"):
        eng.generateBatch([[1, 2], []], maxNewTokens=4)
    with pytest.raises(P.MllmError, match="out of range"):
        eng.generateBatch([[1, 2], [3, 600]], maxNewTokens=4)
    # the handle keeps working
    q = pkg().seeded_prompt(6, 512, 80)
    res, _ = eng.generateBatch([q], maxNewTokens=6, eosId=-1)
    assert res[0]["generatedIds"] == om.generate(q, 6, eos=-1)["generatedIds"]


@pytest.mark.gpu
def test_chunked_forward_rows(cuda_ok):
    """Multi-token forwards split over 16-row forwards: prompt logits and verify rows at pos0 > 0."""
    data = _data("ref-llama")
    eng = _engine(data, env={"MLLM_LWE_TOKENS": "16"})
    om = O.OracleModel(data)
    V = eng.cfg["vocabSize"]
    ids = pkg().seeded_prompt(60, V, 81)
    g = eng.forwardPrompt(ids[:37])
    r = om.forward_prompt(ids[:37])
    assert np.abs(g - r).max() <= LOGIT_TOL
    g, am = eng.forward(ids[37:60], 37, logits_each=True)
    r = om.forward(ids[37:60], 37, logits_each=True)
    assert np.abs(g - r).max() <= LOGIT_TOL
    assert am.tolist() == [int(np.argmax(x)) for x in r]
    eng.destroy()


@pytest.mark.gpu
def test_more_query_heads_than_the_token_batch_engine_takes(cuda_ok):
    """6 query heads per kv head (above the token-batch engine's 4): prefill and multi-token forwards run
    on the persistent decode_kernel, greedy decode on decode1_kernel; streams and logits as the oracle's,
    and generateBatch is refused as unsupported."""
    P = pkg()
    data = P.synthetic_pgw("tiny-llama-r6", 5)
    eng = _engine(data)
    om = O.OracleModel(data)
    try:
        ids = P.seeded_prompt(21, eng.cfg["vocabSize"], 82)
        assert eng.generate(ids, maxNewTokens=20, eosId=-1)["generatedIds"] == om.generate(ids, 20, eos=-1)["generatedIds"]
        g = eng.forwardPrompt(ids)
        assert np.abs(g - om.forward_prompt(ids)).max() <= LOGIT_TOL
        g, am = eng.forward(ids[5:17], 5, logits_each=True)
        r = om.forward(ids[5:17], 5, logits_each=True)
        assert np.abs(g - r).max() <= LOGIT_TOL
        with pytest.raises(P.MllmError):
            eng.generateBatch([ids, ids], maxNewTokens=4, eosId=-1)
    finally:
        eng.destroy()


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["graph", "plain", "persistent"])
def test_speculation_paths(cuda_ok, case):
    """Prompt-lookup speculation (engine/webgpu.js:1164-1282) on the token-batch engine (graph replays,
    plain launches) and on the persistent kernel (a file with 6 query heads per kv head): ids, specHits
    and specTries equal the oracle's."""
    env = {"MLLM_LWE_GRAPH": "0"} if case == "plain" else {}
    data = pkg().synthetic_pgw("tiny-llama-r6", 5) if case == "persistent" else _data("tiny-llama")
    eng = _engine(data, env=env)
    om = O.OracleModel(data)
    ids = pkg().copy_span_prompt(96, 512, 83)
    for k in (2, 4):
        g = eng.generate(ids, maxNewTokens=40, eosId=-1, specK=k, ngram=3)
        r = om.generate_spec(ids, 40, eos=-1, spec_k=k, ngram=3)
        assert g["generatedIds"] == r["generatedIds"]
        assert (g["specHits"], g["specTries"]) == (r["specHits"], r["specTries"])
    # EOS inside an accepted run stops the stream there
    full = om.generate(ids, 40, eos=-1)["generatedIds"]
    eos = full[9]
    g = eng.generate(ids, maxNewTokens=40, eosId=eos, specK=4, ngram=3)
    r = om.generate_spec(ids, 40, eos=eos, spec_k=4, ngram=3)
    assert g["generatedIds"] == r["generatedIds"] and g["stopReason"] == r["stopReason"] == "eos"
    eng.destroy()


@pytest.mark.gpu
@pytest.mark.parametrize("kv_len", [11, 13, 14, 15])
def test_batch_with_cache_lengths_off_the_vector_width(cuda_ok, kv_len):
    """Cache lengths where rep x kv_len is not a multiple of 4 (tiny-llama: 3 query heads per kv head):
    the attention kernel's per-head score rows then end off a 16-byte boundary, and the reduction buffer
    after them must still take float4 stores.  8-token prompts with 3 new ids, against the oracle."""
    data = _data("tiny-llama")
    om = O.OracleModel(data)
    eng = _engine(data, max_slots=16, kv_len=kv_len)
    try:
        V = eng.cfg["vocabSize"]
        seqs = _prompts(V, [8] * 16, 70)
        nnew = min(3, kv_len - 8)
        res, st = eng.generateBatch(seqs, maxNewTokens=nnew, eosId=-1)
        for q, r in zip(seqs, res):
            assert r["generatedIds"] == om.generate(q, nnew, eos=-1)["generatedIds"]
    finally:
        eng.destroy()
