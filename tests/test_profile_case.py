"""Stage-timeline arithmetic of `profile_case.py stages` on a synthetic dump (no device).

The engine dumps `[grid][256]` u64 globaltimer stamps of one forward.  A stage's time is the
difference of the max-over-CTA stamps that close it and the stage before it, and unset stamps (0) are
ignored.
"""
import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "microllm-lab_b200"))
pc = importlib.import_module("profile_case")


def synthetic_dump(grid=4, n_layers=3):
    a = np.zeros((grid, pc.PROF_STAMPS), dtype=np.uint64)
    t = 1_000_000
    a[:, 0] = t
    for l in range(n_layers):
        for k in range(5):
            t += 1000 * (k + 1)  # stage k of every layer: (k + 1) us for the slowest CTA
            a[:, 1 + k + 6 * l] = t - 300 * np.arange(grid)  # other CTAs finish earlier
    a[1:, 1 + 6 * (n_layers - 1)] = 0  # a stamp only CTA 0 wrote (CTAs without QKV rows)
    t += 2000
    a[:, 210] = t
    t += 7000
    a[:, pc.PROF_STAMPS - 3] = t
    t += 500
    a[:, pc.PROF_STAMPS - 2] = t
    return a.reshape(-1)


def test_stage_table_layer_and_tail():
    rows = dict(pc.stage_table(synthetic_dump(), layer=1, n_layers=3))
    for k, name in enumerate(pc.LAYER_STAGES):
        assert rows[name] == pytest.approx(k + 1.0)
    assert rows["per layer"] == pytest.approx(15.0)
    assert rows["wait x2 + final norm"] == pytest.approx(2.0)
    assert rows["lm_head rows + argmax candidates"] == pytest.approx(7.0)
    assert rows["candidate exchange"] == pytest.approx(0.5)
    assert rows["whole forward"] == pytest.approx(3 * 15.0 + 9.5)


def test_stage_table_first_layer_starts_at_the_forward_stamp():
    rows = dict(pc.stage_table(synthetic_dump(), layer=0, n_layers=3))
    assert rows[pc.LAYER_STAGES[0]] == pytest.approx(1.0)


def test_stage_table_rejects_a_layer_that_was_not_stamped():
    with pytest.raises(ValueError):
        pc.stage_table(synthetic_dump(n_layers=2), layer=5, n_layers=6)
