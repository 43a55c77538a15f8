#!/usr/bin/env python3
"""Benchmark of the B200 Q4 decode backend (one JSON line on rank 0).

Default workload = BASELINE config 1: PetitGPT-shaped Q4 model (seed 0), batch 1, 64-token seeded
prompt, 128 greedy new tokens, no speculation, EOS off.  A step is one generate call (prefill + 127
decode steps) in ONE persistent-kernel launch.  ``value`` is generated tokens / device time with the
prompt and output resident in HBM (the reference's tokPerS definition, engine/worker.js:165-176:
tokens over the whole call including prefill); ``e2e`` is the same through the public C-ABI call
with host buffers (H2D prompt, D2H ids inside the timed region).

Multi-GPU (torchrun, one rank per GPU): batch-1 decode does not shard, so every rank runs an
independent replica (its own weights and sequence, prompt seed = rank); value = tokens of all
ranks / max-over-ranks time.  torch.distributed is used only for the barrier and the max.

``--impl reference`` times the CPU restatement of the reference path (oracle/, the JS CPU path of
engine/infer.js; the reference itself needs a JavaScript runtime, absent here) with all host threads
on a bounded sample of the same workload.  Other workloads: ``--workload gemv|gpt2|spec``.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
CACHE = os.environ.get("MLLM_PGW_CACHE", "/tmp/mllm_pgw_cache")
L2_BYTES = 126 * 1024 * 1024

# dram__bytes_read.sum + dram__bytes_write.sum of one decode_kernel launch of the default workload,
# from the ncu capture summarised in profiles/decode_kernel_petitgpt_b1.md (None until captured).
DECODE_TRAFFIC_PER_LAUNCH = None


def pkg():
    return importlib.import_module("microllm-lab_b200")


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def decode_algorithmic_bytes(cfg: dict, n_prompt: int, n_new: int) -> int:
    """Bytes one generate call must move at minimum: every Q4 weight byte and norm gain once per
    forward token step (prefill counted once), K/V rows read per attended position and written once.
    Per decode token at position p: Q4 weights + norms + 2*L*NKV*64*4*(p+1) read + the same per
    position written."""
    d, ff, V, L = cfg["dModel"], cfg["dFf"], cfg["vocabSize"], cfg["nLayers"]
    hd = 64
    kvd = cfg["nKvHeads"] * hd
    q4 = lambda r, c: r * c // 2 + r * (c // 32) * 4
    if cfg["arch"] == "gpt2":
        w = q4(V, d) + L * (q4(3 * d, d) + q4(d, d) + q4(ff, d) + q4(d, ff))
        norms = (L * (4 * d + 3 * d + d + ff + d) + 2 * d) * 4
    else:
        w = q4(V, d) + L * (q4(d + 2 * kvd, d) + q4(d, d) + 2 * q4(ff, d) + q4(d, ff))
        norms = (2 * L + 1) * d * 4
    kv_row = 2 * L * kvd * 4  # K and V of one position over all layers
    total = w + norms + n_prompt * kv_row  # prefill: weights once, K/V written
    for i in range(1, n_new):
        p = n_prompt + i - 1
        total += w + norms + kv_row * (p + 1) + kv_row
    return total


def cpu_baseline_decode(data: bytes, prompt, n_new_full: int, threads: int, sample_decode: int):
    """Oracle (C restatement of engine/infer.js) on a bounded sample: the full prefill plus
    `sample_decode` decode steps; the rate is extrapolated to the full workload."""
    from oracle.oracle import OracleModel
    om = OracleModel(data, threads=threads)
    t0 = time.perf_counter()
    lg = om.forward_prompt(prompt)
    t1 = time.perf_counter()
    tok = int(np.argmax(lg))
    for _ in range(sample_decode):
        tok = int(np.argmax(om.forward_decode(tok)))
    t2 = time.perf_counter()
    per_tok = (t2 - t1) / sample_decode
    full = (t1 - t0) + per_tok * (n_new_full - 1)
    return n_new_full / full, (t1 - t0), per_tok


def batched_algorithmic_bytes(cfg: dict, nseq: int, plen: int, nnew: int, chunks: int) -> int:
    """Minimum bytes of one mllm_generate_batch call: every forward (prefill chunk of tmax tokens, or
    decode step over all sequences) reads the Q4 weights and norms once; every token's K/V row is
    written once; attention reads the K/V rows of positions 0..pos of its own sequence.  `chunks` =
    prefill forwards of the call."""
    d, ff, V, L = cfg["dModel"], cfg["dFf"], cfg["vocabSize"], cfg["nLayers"]
    kvd = cfg["nKvHeads"] * 64
    q4 = lambda r, c: r * c // 2 + r * (c // 32) * 4
    w = q4(V, d) + L * (q4(d + 2 * kvd, d) + q4(d, d) + 2 * q4(ff, d) + q4(d, ff)) + (2 * L + 1) * d * 4
    kv_row = 2 * L * kvd * 4
    total = chunks * w + nseq * plen * kv_row + nseq * kv_row * plen * (plen + 1) // 2
    for i in range(1, nnew):
        pos = plen + i - 1
        total += w + nseq * (kv_row * (pos + 1) + kv_row)
    return total


def cpu_baseline_batched(data: bytes, plen: int, nnew: int, nseq: int, threads: int, sample_decode: int = 4):
    """Oracle on a bounded sample of config 5: one sequence (128-token prefill + `sample_decode` decode
    steps, all host threads inside each forward), extrapolated to nseq sequences x nnew tokens run one
    after another."""
    from oracle.oracle import OracleModel
    om = OracleModel(data, threads=threads)
    prompt = pkg().seeded_prompt(plen, 49152, 4000)
    t0 = time.perf_counter()
    lg = om.forward_prompt(prompt)
    t1 = time.perf_counter()
    tok = int(np.argmax(lg))
    for _ in range(sample_decode):
        tok = int(np.argmax(om.forward_decode(tok)))
    t2 = time.perf_counter()
    per_tok = (t2 - t1) / sample_decode
    per_seq = (t1 - t0) + per_tok * (nnew - 1)
    return nnew / per_seq, (t1 - t0), per_tok


BATCHED = dict(model="smollm2-135m", seed=4, nseq=256, plen=128, nnew=256)


def run_batched_leg(torch, P, local: int, rank: int, ws: int, dist, steps: int, warmup: int, cpu: bool):
    """BASELINE config 5 on this rank's GPU: 256 independent sequences (this rank's partition of the
    global set: sequence ids rank*256 ..), 128-token seeded prompts, 256 greedy new tokens, one
    mllm_generate_batch call per step.  Returns the sub-object for the JSON line (rank 0)."""
    B = BATCHED
    cfg = P.CONFIGS[B["model"]]
    data = P.synthetic_pgw(B["model"], B["seed"], cache_dir=CACHE)
    nseq, plen, nnew = B["nseq"], B["plen"], B["nnew"]
    seqs = [P.seeded_prompt(plen, cfg["vocabSize"], 4000 + rank * nseq + i) for i in range(nseq)]
    eng = P.CudaPetitGPT(data, device=local, max_slots=nseq, kv_len=plen + nnew)
    stream = torch.cuda.Stream()
    eng.set_stream(stream.cuda_stream)
    for _ in range(warmup):
        eng.generateBatch(seqs, maxNewTokens=nnew, eosId=-1)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev_ms, wall_ms, dev_ms, pre_ms, launches, chunks = 0.0, 0.0, [], [], 0, 1
    with ClockSampler(local) as clk:
        for _ in range(steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            t0 = time.perf_counter()
            res, st = eng.generateBatch(seqs, maxNewTokens=nnew, eosId=-1)
            wall_ms += (time.perf_counter() - t0) * 1e3
            e1.record(stream)
            e1.synchronize()
            ev_ms += e0.elapsed_time(e1)
            dev_ms.append(st["deviceMs"])
            pre_ms.append(st["prefillMs"])
            launches += st["kernelLaunches"]
            chunks = st["prefillForwards"]
            assert st["totalGenerated"] == nseq * nnew
    if dist:
        t = torch.tensor([ev_ms, wall_ms], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ev_ms, wall_ms = float(t[0]), float(t[1])
    tokens = nseq * nnew * steps * ws
    hbm, _, peak_kind = peaks()
    alg = batched_algorithmic_bytes(cfg, nseq, plen, nnew, chunks)
    ms = ev_ms / steps
    achieved = alg / (ms / 1e3) / 1e9
    out = {
        "metric": "replicated multi-sequence decode aggregate tok/s (SmolLM2-135M shape, 256 seqs/GPU, "
                  "128-token prompts, 256 new tokens)",
        "value": tokens / (ev_ms / 1e3), "unit": "tok/s", "n_gpus": ws, "steps": steps, "warmup": warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "config": {"workload": "config5 smollm2-135m 256 seqs/GPU p128 n256", "sequences_per_gpu": nseq,
                   "partition": "sequence ids rank*256 .. rank*256+255", "inputs": "larger than L2 (4.5 GB KV)",
                   "timing": "CUDA events around one mllm_generate_batch call (its 128 KB prompt upload and "
                             "256 KB id download included)"},
        "prefill_ms": float(np.mean(pre_ms)), "decode_tok_s_per_gpu": nseq * (nnew - 1) / ((np.mean(dev_ms) - np.mean(pre_ms)) / 1e3),
        "e2e": {"value": tokens / (wall_ms / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": nseq * plen * 4 + (3 * nseq * plen + 2 * nseq) * 4 + nseq * 4,
                "d2h_bytes_per_step": nseq * nnew * 4 + nseq * 4 + 17 * 4},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": peak_kind, "traffic": None, "kernel": "whole call (token-batch kernels; attention "
                     "over the fp32 KV cache dominates)", "algorithmic_bytes_per_step": alg},
        "clocks": clk.summary(),
    }
    if cpu and rank == 0 and ws == 1:
        threads = os.cpu_count() or 1
        v, pre, per = cpu_baseline_batched(data, plen, nnew, nseq, threads)
        out["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                               "sample": f"oracle, {threads} threads inside each forward: one sequence's 128-token "
                                         f"prefill ({pre:.2f} s) + 4 decode steps ({per*1e3:.0f} ms/token), "
                                         f"extrapolated to 256 sequences x 256 tokens run in turn"}
    eng.destroy()
    return out


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def run_reference(args):
    """--impl reference: the CPU restatement of the reference path, all host threads, rank 0 only."""
    ws, rank, _ = dist_setup()
    if rank != 0:
        return
    P = pkg()
    cfg = P.CONFIGS["petitgpt"]
    data = P.synthetic_pgw("petitgpt", 0, cache_dir=CACHE)
    prompt = P.seeded_prompt(64, cfg["vocabSize"], 0)
    threads = os.cpu_count() or 1
    sample = 4
    for _ in range(args.warmup):
        cpu_baseline_decode(data, prompt, 128, threads, sample)
    vals, pre, per = [], [], []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, a, b = cpu_baseline_decode(data, prompt, 128, threads, sample)
        vals.append(v)
        pre.append(a)
        per.append(b)
    wall = time.perf_counter() - t0
    v = float(np.mean(vals))
    line = {
        "impl": "reference", "metric": "batch-1 Q4 decode tok/s (PetitGPT shape, 64-token prompt, 128 new tokens)",
        "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": wall / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f64-accumulate/f32-store", "data": "synthetic (seeded N(0,0.02) Q4 weights, seeded prompt)",
        "config": {"workload": "config1 petitgpt b1 p64 n128", "model": "PetitGPT-shaped Q4 (30L d576 9/3 ff1536 V32000)",
                   "global_batch": 1, "seq_len": 192, "parallelism": "replicas"},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"per step: 64-token prefill + {sample} decode steps, extrapolated to 127 "
                                   f"decode steps (prefill {np.mean(pre):.2f} s, {np.mean(per)*1e3:.1f} ms/token)"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_decode(args):
    import torch
    ws, rank, local = dist_setup()
    dist = None
    if ws > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    P = pkg()
    name = "petitgpt"
    cfg = P.CONFIGS[name]
    data = P.synthetic_pgw(name, 0, cache_dir=CACHE)
    n_prompt, n_new = 64, 128
    prompt = P.seeded_prompt(n_prompt, cfg["vocabSize"], rank)
    eng = P.CudaPetitGPT(data, device=local)
    stream = torch.cuda.Stream()
    eng.set_stream(stream.cuda_stream)
    d_ids = torch.from_numpy(prompt).to(f"cuda:{local}")
    d_out = torch.zeros(n_new + 16, dtype=torch.int32, device=f"cuda:{local}")
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=f"cuda:{local}")
    h_prompt = torch.from_numpy(prompt).pin_memory()
    h_out = torch.zeros(n_new + 16, dtype=torch.int32).pin_memory()

    launches = [0]

    def step_device():
        st = eng.generate_device(d_ids.data_ptr(), n_prompt, d_out.data_ptr(), n_new, -1)
        assert st.n_generated == n_new, st.n_generated
        launches[0] += st.kernel_launches
        return st

    def step_e2e():
        import ctypes
        st = P.engine.Stats()
        eng._check(eng._lib.mllm_generate(eng._h, 0, ctypes.c_void_p(h_prompt.data_ptr()), n_prompt, n_new, -1, 0, 3,
                                          ctypes.c_void_p(h_out.data_ptr()), ctypes.byref(st)))
        assert st.n_generated == n_new

    def timed(fn, k):
        """k steps, each bracketed by events on the launch stream, L2 flushed before each step."""
        total = 0.0
        dev_ms = []
        for _ in range(k):
            with torch.cuda.stream(stream):
                flush.fill_(1.0)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                st = fn()
                e1.record(stream)
            e1.synchronize()
            total += e0.elapsed_time(e1)
            if st is not None:
                dev_ms.append(st.total_ms)
        return total, dev_ms

    for _ in range(args.warmup):
        step_device()
        step_e2e()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    launches[0] = 0
    with ClockSampler(local) as clk:
        t_dev, dev_ms = timed(step_device, args.steps)
        torch.cuda.synchronize()
        t_e2e, _ = timed(step_e2e, args.steps)
    torch.cuda.synchronize()
    if dist:
        t = torch.tensor([t_dev, t_e2e], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_dev, t_e2e = float(t[0]), float(t[1])
        dist.barrier()
    tokens = n_new * args.steps * ws
    value = tokens / (t_dev / 1e3)
    e2e = tokens / (t_e2e / 1e3)
    ms_step = t_dev / args.steps
    hbm, _, peak_kind = peaks()
    alg = decode_algorithmic_bytes(cfg, n_prompt, n_new)
    achieved = alg / (ms_step / 1e3) / 1e9
    line = {
        "metric": "batch-1 Q4 decode tok/s (PetitGPT shape, 64-token prompt, 128 new tokens)",
        "value": value, "unit": "tok/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q4xf32",
        "data": "synthetic (seeded N(0,0.02) Q4 weights, seeded uniform prompt ids; real checkpoints are LFS stubs)",
        "config": {"workload": "config1 petitgpt b1 p64 n128", "model": "PetitGPT-shaped Q4 (30L d576 9/3 ff1536 V32000)",
                   "global_batch": ws, "seq_len": n_prompt + n_new, "parallelism": f"replicas x{ws}",
                   "l2": "flushed (256 MB write) before every timed step; weights 78 MB fit in L2 within a step",
                   "tokens_per_step": n_new,
                   "launches_per_step": launches[0] // max(args.steps, 1),
                   "path": "prefill as token-batch tensor-core forwards, then the 127 decode steps in one "
                           "persistent single-token kernel launch"},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": n_prompt * 4, "d2h_bytes_per_step": n_new * 4 + 68},
        "gpu_launches": launches[0],
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": peak_kind, "traffic": DECODE_TRAFFIC_PER_LAUNCH,
                     "kernel": "decode1_kernel<3,6> (whole generate call)", "algorithmic_bytes_per_launch": alg,
                     "kernel_ms_device_timer": float(np.mean(dev_ms)) if dev_ms else None},
        "clocks": clk.summary(),
    }
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        v, pre, per = cpu_baseline_decode(data, prompt, n_new, 1, 4)
        line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": 1, "kind": "port",
                                "sample": f"oracle (C restatement of engine/infer.js), 1 thread: 64-token prefill "
                                          f"({pre:.2f} s) + 4 decode steps ({per*1e3:.0f} ms/token), extrapolated "
                                          f"to 127 decode steps"}
    eng.destroy()
    if not args.no_batched:
        line["batched"] = run_batched_leg(torch, P, local, rank, ws, dist, args.batched_steps, 1,
                                          not args.no_cpu_baseline)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batched", action="store_true", help="skip the config-5 batched sub-object")
    ap.add_argument("--batched-steps", type=int, default=3)
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_decode(args)


if __name__ == "__main__":
    main()
