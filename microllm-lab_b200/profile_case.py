"""Small, fixed cases of each decode path, sized for a profiler capture.

Usage (from the repository root):

    python microllm-lab_b200/profile_case.py decode [--model petitgpt] [--prompt 64] [--new 24]
    python microllm-lab_b200/profile_case.py spec   [--model smollm2-360m] [--prompt 512] [--new 64] [--k 4]
    python microllm-lab_b200/profile_case.py batch  [--seqs 256] [--prompt 255] [--kv 384] [--new 3]
    python microllm-lab_b200/profile_case.py gemv   [--rows 49152] [--cols 576] [--m 1]
    python microllm-lab_b200/profile_case.py stages [--model petitgpt] [--forward 20] [--layer 15]

Each case builds a seeded synthetic model (the same generators the tests and `bench.py` use), runs
the path once and prints one summary line. Nothing is timed here: the cases exist so that a launch
list or a full capture of one kernel can be taken on a workload small enough to end quickly.
`MLLM_PROFILE_DECODE_STEPS` / `MLLM_PROFILE_SPEC_ITERS` (read by the engine) bracket the first decode
steps or speculation iterations with cudaProfilerStart/Stop, for `--profile-from-start off`.

`stages` runs the decode case with the single-token kernel's stage timestamps switched on
(`MLLM_STAGE_PROFILE=<forward>`, dumped by the engine as raw u64 `[grid][256]` globaltimer values) and
prints, for one layer of that forward, each stage's time as the difference of the max-over-CTA stamps
that close it and the previous stage, then the lm_head tail.
"""
import argparse
import importlib
import os
import sys
import tempfile

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)


PROF_STAMPS = 256  # stamps per CTA in the dump
LAYER_STAGES = ["wait x2 + norm1 + QKV rows", "attention (head CTAs)", "proj rows + residual (x1)",
                "wait x1 + norm2 + w1/w3 rows", "w2 rows + residual (x2)"]


def stage_table(dump, layer: int, n_layers: int):
    """(name, us) rows from a stage dump: stamp 1 + k + 6 l closes stage k of layer l, stamp 0 opens the
    forward, 210 / PROF_STAMPS - 3 / PROF_STAMPS - 2 close the final norm, the lm_head rows and the
    candidate exchange.  Each time is the difference of max-over-CTA stamps (unset stamps are 0)."""
    import numpy as np
    a = np.asarray(dump, dtype=np.uint64).reshape(-1, PROF_STAMPS).astype(np.int64)
    tmax = np.where(a > 0, a, -1).max(axis=0)

    def at(i):
        if tmax[i] < 0:
            raise ValueError(f"stamp {i} was not written (forward or layer out of range?)")
        return int(tmax[i])

    rows = []
    prev = at(0) if layer == 0 else at(5 + 6 * (layer - 1))
    for k, name in enumerate(LAYER_STAGES):
        cur = at(1 + k + 6 * layer)
        rows.append((name, (cur - prev) / 1e3))
        prev = cur
    rows.append(("per layer", sum(us for _, us in rows)))
    last = at(5 + 6 * (n_layers - 1))
    rows.append(("wait x2 + final norm", (at(210) - last) / 1e3))
    rows.append(("lm_head rows + argmax candidates", (at(PROF_STAMPS - 3) - at(210)) / 1e3))
    rows.append(("candidate exchange", (at(PROF_STAMPS - 2) - at(PROF_STAMPS - 3)) / 1e3))
    rows.append(("whole forward", (at(PROF_STAMPS - 2) - at(0)) / 1e3))
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("case", choices=["decode", "spec", "batch", "gemv", "stages"])
    ap.add_argument("--forward", type=int, default=20)
    ap.add_argument("--layer", type=int, default=15)
    ap.add_argument("--out", default=os.path.join(tempfile.gettempdir(), "mllm_stage_profile.bin"))
    ap.add_argument("--model", default=None)
    ap.add_argument("--seed", type=int, default=None)
    ap.add_argument("--prompt", type=int, default=None)
    ap.add_argument("--new", type=int, default=None)
    ap.add_argument("--k", type=int, default=4)
    ap.add_argument("--seqs", type=int, default=256)
    ap.add_argument("--kv", type=int, default=384)
    ap.add_argument("--rows", type=int, default=49152)
    ap.add_argument("--cols", type=int, default=576)
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--cache-dir", default="/tmp/mllm_pgw_cache")
    a = ap.parse_args(argv)
    if a.case == "stages":  # read by the engine when it is created
        os.environ["MLLM_STAGE_PROFILE"] = str(a.forward)
        os.environ["MLLM_STAGE_PROFILE_OUT"] = a.out
    P = importlib.import_module("microllm-lab_b200")

    if a.case == "gemv":
        import numpy as np
        import torch
        rng = np.random.default_rng(1)
        w = rng.standard_normal((a.rows, a.cols), dtype=np.float32) * np.float32(0.02)
        packed, scales = P.quant_q4(w)
        pk = torch.from_numpy(np.ascontiguousarray(packed).reshape(-1)).cuda()
        sc = torch.from_numpy(np.ascontiguousarray(scales).reshape(-1)).cuda()
        x = torch.from_numpy(rng.standard_normal((a.m, a.cols), dtype=np.float32)).cuda()
        y = torch.empty((a.m, a.rows), device="cuda")
        flush = torch.empty(64 * 1024 * 1024, device="cuda")  # 256 MB: larger than L2
        for _ in range(3):
            flush.fill_(1.0)
            P.gemv_q4_device(pk.data_ptr(), sc.data_ptr(), x.data_ptr(), y.data_ptr(), a.rows, a.cols, a.m)
        torch.cuda.synchronize()
        print(f"gemv {a.rows}x{a.cols} m={a.m}: 3 launches")
        return

    if a.case == "batch":
        model = a.model or "smollm2-135m"
        data = P.synthetic_pgw(model, 4 if a.seed is None else a.seed, cache_dir=a.cache_dir)
        eng = P.CudaPetitGPT(data, max_slots=a.seqs, kv_len=a.kv)
        plen = 255 if a.prompt is None else a.prompt
        seqs = [P.seeded_prompt(plen, eng.cfg["vocabSize"], 1000 + i) for i in range(a.seqs)]
        _, st = eng.generateBatch(seqs, maxNewTokens=3 if a.new is None else a.new, eosId=-1)
        print(f"batch {model}: {st}")
        return

    if a.case == "stages":
        import numpy as np
        model = a.model or "petitgpt"
        data = P.synthetic_pgw(model, 0 if a.seed is None else a.seed, cache_dir=a.cache_dir)
        eng = P.CudaPetitGPT(data)
        ids = P.seeded_prompt(64 if a.prompt is None else a.prompt, eng.cfg["vocabSize"], 0)
        eng.generate(ids, maxNewTokens=128 if a.new is None else a.new, eosId=-1)
        n_layers = eng.cfg["nLayers"]
        eng.destroy()
        rows = stage_table(np.fromfile(a.out, dtype=np.uint64), a.layer, n_layers)
        print(f"stages {model}: forward {a.forward}, layer {a.layer} (max-over-CTA stamp deltas, us)")
        for name, us in rows:
            print(f"  {name:34s} {us:8.2f}")
        return

    if a.case == "decode":
        model = a.model or "petitgpt"
        data = P.synthetic_pgw(model, 0 if a.seed is None else a.seed, cache_dir=a.cache_dir)
        eng = P.CudaPetitGPT(data)
        ids = P.seeded_prompt(64 if a.prompt is None else a.prompt, eng.cfg["vocabSize"], 0)
        r = eng.generate(ids, maxNewTokens=24 if a.new is None else a.new, eosId=-1)
    else:
        model = a.model or "smollm2-360m"
        data = P.synthetic_pgw(model, 3 if a.seed is None else a.seed, cache_dir=a.cache_dir)
        eng = P.CudaPetitGPT(data)
        ids = P.copy_span_prompt(512 if a.prompt is None else a.prompt, eng.cfg["vocabSize"], 3)
        r = eng.generate(ids, maxNewTokens=64 if a.new is None else a.new, eosId=-1, specK=a.k, ngram=3)
    print(f"{a.case} {model}: deviceMs {r['deviceMs']:.3f} forwards {r['forwards']} "
          f"specHits {r['specHits']} specTries {r['specTries']} kernelLaunches {r['kernelLaunches']}")


if __name__ == "__main__":
    main()
