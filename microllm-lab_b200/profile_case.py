"""Small, fixed cases of each decode path, sized for a profiler capture.

Usage (from the repository root):

    python microllm-lab_b200/profile_case.py decode [--model petitgpt] [--prompt 64] [--new 24]
    python microllm-lab_b200/profile_case.py spec   [--model smollm2-360m] [--prompt 512] [--new 64] [--k 4]
    python microllm-lab_b200/profile_case.py batch  [--seqs 256] [--prompt 255] [--kv 384] [--new 3]
    python microllm-lab_b200/profile_case.py gemv   [--rows 49152] [--cols 576] [--m 1]

Each case builds a seeded synthetic model (the same generators the tests and `bench.py` use), runs
the path once and prints one summary line. Nothing is timed here: the cases exist so that a launch
list or a full capture of one kernel can be taken on a workload small enough to end quickly.
`MLLM_PROFILE_DECODE_STEPS` / `MLLM_PROFILE_SPEC_ITERS` (read by the engine) bracket the first decode
steps or speculation iterations with cudaProfilerStart/Stop, for `--profile-from-start off`.
"""
import argparse
import importlib
import os
import sys

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("case", choices=["decode", "spec", "batch", "gemv"])
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
