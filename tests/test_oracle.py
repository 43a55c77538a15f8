"""The CPU oracle (C restatement of engine/infer.js) pinned against HF transformers float64 forwards
of models written by the reference's own converters, plus unit cases of the control-flow pieces."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, pkg
from oracle import oracle as O


def _ref(name):
    return open(os.path.join(GOLDEN, name), "rb").read()


def test_oracle_llama_matches_hf_float64():
    z = np.load(os.path.join(GOLDEN, "ref_llama_hf.npz"))
    om = O.OracleModel(_ref("ref_llama.pgw"))
    lg = om.forward_prompt(z["prompt"])
    np.testing.assert_allclose(lg, z["last_logits"], atol=2e-5, rtol=0)
    out = om.generate(z["prompt"], len(z["greedy"]), eos=-1, step_logits=True)
    assert out["generatedIds"] == z["greedy"].tolist()
    np.testing.assert_allclose(out["stepLogits"], z["step_logits"], atol=5e-5, rtol=0)


def test_oracle_gpt2_matches_hf_float64():
    """GPT-2 path incl. SmoothQuant scale_factors (engine/infer.js:416-419), wpe, LN, biases, GELU."""
    z = np.load(os.path.join(GOLDEN, "ref_gpt2_hf.npz"))
    om = O.OracleModel(_ref("ref_gpt2.pgw"))
    prompt = z["prompt"]
    for t in range(1, len(prompt) + 1):
        lg = om.forward_prompt(prompt[:t])
        np.testing.assert_allclose(lg, z["logits"][t - 1], atol=5e-5, rtol=0, err_msg=f"t={t}")


def test_oracle_decode_equals_prompt_forward():
    """forwardDecode after forwardPrompt == forwardPrompt of the longer prompt (f64 math, exact)."""
    P = pkg()
    om = O.OracleModel(P.synthetic_pgw("tiny-llama", 3))
    ids = P.seeded_prompt(9, 512, 1)
    om.forward_prompt(ids[:8])
    a = om.forward_decode(int(ids[8]))
    b = om.forward_prompt(ids)
    np.testing.assert_array_equal(a, b)


def test_gemv_variants():
    rng = np.random.default_rng(0)
    P = pkg()
    w = rng.standard_normal((40, 96), dtype=np.float32) * np.float32(0.02)
    packed, sc = P.quant_q4(w)
    x = rng.standard_normal(96, dtype=np.float32)
    y = O.gemv_q4(packed, sc, x)
    ref = P.dequant_q4(packed, sc).astype(np.float64) @ x.astype(np.float64)
    np.testing.assert_allclose(y, ref.astype(np.float32), rtol=1e-6, atol=1e-7)
    y32 = O.gemv_q4_f32acc(packed, sc, x)
    np.testing.assert_allclose(y32, y, rtol=1e-4, atol=1e-6)
    y8 = O.gemv_q4(packed, sc, x, threads=4)
    np.testing.assert_array_equal(y8, y)


def test_lookup_draft_cases():
    """engine/webgpu.js:846-865: latest earlier n-gram match, continuation truncated at the end."""
    assert O.lookup_draft([1, 2, 3], 2, 3) == []                      # len < n + 1
    assert O.lookup_draft([5, 1, 2, 3, 9, 1, 2, 3], 2, 3) == [9, 1]
    assert O.lookup_draft([1, 2, 3, 7, 1, 2, 3, 8, 1, 2, 3], 4, 3) == [8, 1, 2, 3]  # latest match wins
    assert O.lookup_draft([1, 2, 3, 1, 2, 3], 5, 3) == [1, 2, 3]     # continuation hits the end
    assert O.lookup_draft([4, 4, 4, 4], 2, 3) == [4]                  # overlapping match at i = 0
    assert O.lookup_draft([1, 2, 3, 4, 5, 6], 2, 3) == []             # no match


def test_argmax_gpt2_penalties():
    """engine/infer.js:252-287: 3-gram ban and 1.15 repetition penalty on the last 32 ids."""
    lg = np.zeros(10, np.float32)
    lg[[2, 5, 7]] = [1.0, 1.1, -0.5]
    assert O.argmax_gpt2(lg, []) == 5
    assert O.argmax_gpt2(lg, [5]) == 2          # 1.1 / 1.15 < 1.0
    assert O.argmax_gpt2(lg, [1, 5, 1, 5]) == 2
    # ban: history has (3, 4) -> 5 and ends with (3, 4): 5 is banned
    assert O.argmax_gpt2(lg, [3, 4, 5, 3, 4]) == 2
    lg2 = np.full(4, -1.0, np.float32)
    assert O.argmax_gpt2(lg2, [0]) == 1         # negative logits get multiplied
    # ties keep the lowest index
    assert O.argmax_gpt2(np.ones(6, np.float32), []) == 0


def test_generate_stop_rules():
    """EOS stop, prompt truncation (infer.js:604-608) and the maxSeqLen stop (infer.js:626)."""
    P = pkg()
    data = P.synthetic_pgw("tiny-llama", 5)
    om = O.OracleModel(data)
    ids = P.seeded_prompt(12, 512, 2)
    full = om.generate(ids, 10, eos=-1)
    assert len(full["generatedIds"]) == 10 and full["stopReason"] == "max_new_tokens"
    eos = full["generatedIds"][3]
    first = full["generatedIds"].index(eos)
    r = om.generate(ids, 10, eos=eos)
    assert r["generatedIds"] == full["generatedIds"][:first + 1] and r["stopReason"] == "eos"
    # maxSeqLen 160: a 150-id prompt with 20 new ids is cut to 139 ids
    long = P.seeded_prompt(150, 512, 4)
    r = om.generate(long, 20, eos=-1)
    assert len(r["generatedIds"]) == 20
    ref = om.generate(long[-139:], 20, eos=-1)
    assert r["generatedIds"] == ref["generatedIds"]


def test_spec_generate_equals_greedy():
    """With f64 math the verify forward equals sequential decode, so speculation returns the greedy stream."""
    P = pkg()
    data = P.synthetic_pgw("tiny-llama", 9)
    om = O.OracleModel(data)
    ids = P.copy_span_prompt(96, 512, 7)
    g = om.generate(ids, 40, eos=-1)
    for k in (2, 4, 8):
        s = om.generate_spec(ids, 40, eos=-1, spec_k=k, ngram=3)
        assert s["generatedIds"] == g["generatedIds"], k
        assert s["specTries"] == s["forwards"]
        assert len(s["generatedIds"]) == s["forwards"] + 1 + s["specHits"]


def _js_gemv_row(wrow, x, conv):
    """One row of gemvF32 / gemvF16 / gemvBf16 / gemvQ8 as the JS loops write it (engine/infer.js:10-86):
    a double accumulator, gemvF32's 8-way unrolled body and tail loop, per-element conversion."""
    n = len(x)
    s = 0.0
    k = 0
    while k < n - 7:
        for j in range(8):
            s += float(conv(wrow[k + j])) * float(x[k + j])
        k += 8
    while k < n:
        s += float(conv(wrow[k])) * float(x[k])
        k += 1
    return s


def test_gemv_dense_oracle_matches_the_js_loops():
    """The vectorised dense / q8 GEMV oracle against a scalar restatement of the JS row loops, including
    f16 subnormals and infinities-free extremes, bf16 bit patterns and negative int8."""
    rng = np.random.default_rng(5)
    rows, cols = 6, 44
    x = rng.standard_normal(cols).astype(np.float32)
    f32 = (rng.standard_normal((rows, cols)) * 0.05).astype(np.float32)
    f16 = (rng.standard_normal((rows, cols)) * 0.05).astype(np.float16)
    f16[0, :4] = np.array([6e-8, -3e-6, 65504.0, -0.0], np.float16)  # subnormal, tiny, largest finite
    f16w = f16.view(np.uint16)
    bf = rng.integers(0, 1 << 16, size=(rows, cols), dtype=np.uint16)
    bf[(bf & 0x7F80) == 0x7F80] &= 0xBFFF  # no inf / nan patterns
    q8 = rng.integers(-128, 128, size=(rows, cols)).astype(np.int8)
    sc = (rng.random(rows) * 0.01).astype(np.float32)
    cases = [("f32", f32, None, lambda v: np.float32(v)),
             ("f16", f16w, None, lambda v: np.uint16(v).view(np.float16).astype(np.float32)),
             ("bf16", bf, None, lambda v: np.array([np.uint32(v) << np.uint32(16)], np.uint32).view(np.float32)[0]),
             ("q8", q8, sc, lambda v: np.float32(v))]
    for dt, w, s, conv in cases:
        got = O.gemv_dense(dt, w, s, x)
        for r in range(rows):
            want = _js_gemv_row(w[r], x, conv)
            if dt == "q8":
                want *= float(s[r])
            assert np.float32(want) == got[r] or abs(float(got[r]) - want) <= 1e-6 * max(1.0, abs(want)), (dt, r)

