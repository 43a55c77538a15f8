"""Persistent decode kernel (libmllm_cuda.so, through the C ABI) against the CPU oracle.

Bars (the build's stated tolerances): token ids, drafts/accept counts and greedy streams bit-exact;
logits max-abs <= 2e-2 against the f64-accumulating oracle (fp32 accumulation on the device)."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, pkg
from oracle import oracle as O

LOGIT_TOL = 2e-2


def _models():
    P = pkg()
    return {
        "tiny-llama": P.synthetic_pgw("tiny-llama", 3),
        "tiny-gpt2": P.synthetic_pgw("tiny-gpt2", 4),
        "ref-llama": open(os.path.join(GOLDEN, "ref_llama.pgw"), "rb").read(),
        "ref-gpt2": open(os.path.join(GOLDEN, "ref_gpt2.pgw"), "rb").read(),
    }


@pytest.fixture(scope="module")
def models(cuda_ok):
    P = pkg()
    out = {}
    for k, data in _models().items():
        out[k] = (data, P.CudaPetitGPT(data), O.OracleModel(data))
    yield out
    for _, eng, _ in out.values():
        eng.destroy()


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["tiny-llama", "tiny-gpt2", "ref-llama", "ref-gpt2"])
def test_forward_prompt_logits(models, name):
    data, eng, om = models[name]
    V = eng.cfg["vocabSize"]
    ids = pkg().seeded_prompt(7, V, 11)
    g = eng.forwardPrompt(ids)
    r = om.forward_prompt(ids)
    err = np.abs(g - r).max()
    assert err <= LOGIT_TOL, err
    assert eng.cacheLen == 7
    assert int(np.argmax(g)) == int(np.argmax(r))


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["tiny-llama", "tiny-gpt2"])
def test_decode_steps(models, name):
    data, eng, om = models[name]
    V = eng.cfg["vocabSize"]
    ids = pkg().seeded_prompt(5, V, 12)
    g = eng.forwardPrompt(ids)
    r = om.forward_prompt(ids)
    tok = int(np.argmax(r))
    for step in range(12):
        assert int(np.argmax(g)) == tok
        g = eng.forwardDecode(tok)
        r = om.forward_decode(tok)
        assert np.abs(g - r).max() <= LOGIT_TOL, step
        tok = int(np.argmax(r))
    assert eng.cacheLen == om.cache_len == 5 + 12


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["tiny-llama", "ref-llama"])
def test_verify_forward_each_row(models, name):
    """The verify forward (engine/webgpu.js:1248): logits and argmax for every row, at pos0 > 0."""
    data, eng, om = models[name]
    V = eng.cfg["vocabSize"]
    ids = pkg().seeded_prompt(20, V, 13)
    eng.forwardPrompt(ids[:11])
    om.forward_prompt(ids[:11])
    g, am = eng.forward(ids[11:20], 11, logits_each=True)
    r = om.forward(ids[11:20], 11, logits_each=True)
    assert g.shape == r.shape == (9, V)
    assert np.abs(g - r).max() <= LOGIT_TOL
    assert am.tolist() == [int(np.argmax(x)) for x in r]


@pytest.mark.gpu
def test_prefill_longer_than_one_forward(models):
    """Prompts longer than the kernel's tokens-per-forward run as several chunks in one launch."""
    data, eng, om = models["tiny-llama"]
    ids = pkg().seeded_prompt(100, 512, 14)
    assert eng.maxTokensPerForward < 100
    g = eng.forwardPrompt(ids)
    r = om.forward_prompt(ids)
    assert np.abs(g - r).max() <= LOGIT_TOL


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["tiny-llama", "tiny-gpt2", "ref-llama", "ref-gpt2"])
def test_generate_matches_oracle(models, name):
    """engine/infer.js:603-646 greedy stream (GPT-2: penalised argmax) bit-exact."""
    data, eng, om = models[name]
    V = eng.cfg["vocabSize"]
    ids = pkg().seeded_prompt(16, V, 15)
    g = eng.generate(ids, maxNewTokens=48, eosId=-1)
    r = om.generate(ids, 48, eos=-1)
    assert g["generatedIds"] == r["generatedIds"]
    assert g["stopReason"] == r["stopReason"] == "max_new_tokens"
    assert len(set(r["generatedIds"])) > 3  # the test model does not sit in a one-token loop


LONG_CFGS = {
    # GQA 3:1 and 6:2, and GPT-2 (no RoPE): contexts of several 128-position attention splits
    "llama-3-1": dict(arch="llama", vocabSize=512, nLayers=2, dModel=192, nHeads=3, nKvHeads=1, dFf=320,
                      maxSeqLen=640, ropeTheta=10000.0),
    "llama-6-2": dict(arch="llama", vocabSize=384, nLayers=2, dModel=384, nHeads=6, nKvHeads=2, dFf=256,
                      maxSeqLen=640, ropeTheta=10000.0),
    "gpt2": dict(arch="gpt2", vocabSize=640, nLayers=2, dModel=128, nHeads=2, nKvHeads=2, dFf=512, maxSeqLen=640),
}


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(LONG_CFGS))
def test_long_context_generate_matches_oracle(cuda_ok, name):
    """Single-token decode past 128, 256, ... positions, where the attention of each head is split over
    several CTAs and merged: the greedy stream equals the oracle's (prompt 500, 40 new ids)."""
    P = pkg()
    cfg = dict(LONG_CFGS[name])
    data = P.synthetic_pgw(cfg, 21, cache_dir="/tmp/mllm_pgw_cache")
    eng = P.CudaPetitGPT(data)
    try:
        om = O.OracleModel(data)
        ids = P.seeded_prompt(500, cfg["vocabSize"], 22)
        g = eng.generate(ids, maxNewTokens=40, eosId=-1)
        r = om.generate(ids, 40, eos=-1)
        assert g["generatedIds"] == r["generatedIds"]
        # one single-token forward at position 300 (three splits), logits against the oracle
        eng.resetCache()
        eng.forwardPrompt(ids[:300])
        lg = eng.forwardDecode(int(ids[300]))
        om2 = O.OracleModel(data)
        om2.forward_prompt(ids[:300])
        ref = om2.forward_decode(int(ids[300]))
        assert np.max(np.abs(np.asarray(lg) - ref)) <= 2e-2
    finally:
        eng.destroy()


@pytest.mark.gpu
@pytest.mark.parametrize("k", [2, 4, 8])
def test_speculative_generate_matches_oracle(models, k):
    """engine/webgpu.js:1164-1282 with lookupDraft: tokens, accepted-draft count and tries bit-exact."""
    data, eng, om = models["tiny-llama"]
    ids = pkg().copy_span_prompt(96, 512, 16)
    g = eng.generate(ids, maxNewTokens=40, eosId=-1, specK=k, ngram=3)
    r = om.generate_spec(ids, 40, eos=-1, spec_k=k, ngram=3)
    assert g["generatedIds"] == r["generatedIds"]
    assert (g["specHits"], g["specTries"]) == (r["specHits"], r["specTries"])
    greedy = om.generate(ids, 40, eos=-1)
    assert g["generatedIds"] == greedy["generatedIds"]


@pytest.mark.gpu
def test_generate_stop_rules(models):
    data, eng, om = models["tiny-llama"]
    ids = pkg().seeded_prompt(12, 512, 17)
    full = om.generate(ids, 12, eos=-1)["generatedIds"]
    eos = full[5]
    g = eng.generate(ids, maxNewTokens=12, eosId=eos)
    r = om.generate(ids, 12, eos=eos)
    assert g["generatedIds"] == r["generatedIds"] and g["stopReason"] == "eos"
    # maxNewTokens = 1: prefill only
    assert eng.generate(ids, maxNewTokens=1, eosId=-1)["generatedIds"] == full[:1]
    # maxSeqLen 160: the prompt is cut to maxSeq - maxNew - 1 ids (engine/infer.js:604-608)
    long = pkg().seeded_prompt(150, 512, 18)
    g = eng.generate(long, maxNewTokens=20, eosId=-1)
    assert g["generatedIds"] == om.generate(long, 20, eos=-1)["generatedIds"]
    # single-token prompt
    assert eng.generate(ids[:1], maxNewTokens=8, eosId=-1)["generatedIds"] == om.generate(ids[:1], 8, eos=-1)["generatedIds"]


@pytest.mark.gpu
def test_argument_errors(models):
    P = pkg()
    data, eng, om = models["tiny-llama"]
    with pytest.raises(P.MllmError, match="out of range"):
        eng.generate([1, 2, 600], maxNewTokens=4)
    with pytest.raises(P.MllmError):
        eng.forward([1, 2], pos0=eng.cacheLen + 5)
    with pytest.raises(P.MllmError):
        eng.forward([1], pos0=eng.kvLen)
    with pytest.raises(P.MllmError):
        eng.generate([], maxNewTokens=4)


@pytest.mark.gpu
def test_device_wait_limit_reports_timeout_and_recovers(models):
    """Failure detection without a fault: every CTA waits on a word nothing writes; the 50 ms limit
    runs out, the call returns MLLM_ERR_TIMEOUT, and the same handle then generates correctly."""
    data, eng, om = models["tiny-llama"]
    assert eng.selftest_timeout(50) == -6
    ids = pkg().seeded_prompt(10, 512, 19)
    assert eng.generate(ids, maxNewTokens=8, eosId=-1)["generatedIds"] == om.generate(ids, 8, eos=-1)["generatedIds"]


@pytest.mark.gpu
def test_petitgpt_shape_generate(cuda_ok):
    """Full PetitGPT-shaped model (BASELINE config 1 weights, seed 0): 12 greedy ids and the first
    logits row against the oracle."""
    P = pkg()
    data = P.synthetic_pgw("petitgpt", 0, cache_dir="/tmp/mllm_pgw_cache")
    eng = P.CudaPetitGPT(data)
    om = O.OracleModel(data, threads=os.cpu_count() or 1)
    ids = P.seeded_prompt(64, 32000, 0)
    g = eng.generate(ids, maxNewTokens=12, eosId=-1)
    r = om.generate(ids, 12, eos=-1, step_logits=True)
    assert g["generatedIds"] == r["generatedIds"]
    lg = eng.forwardPrompt(ids)
    assert np.abs(lg - r["stepLogits"][0]).max() <= LOGIT_TOL
    eng.destroy()
