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
on a bounded sample of the same workload.  Other workloads: ``--workload gpt2`` (config 3),
``spec4``/``spec8`` (config 4, prompt-lookup speculation), ``gemv`` (config 2).  The default run also
measures config 5 (replicated multi-sequence decode) as the ``batched`` sub-object.
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

# dram__bytes_read.sum + dram__bytes_write.sum of ONE decode1_kernel launch of the config-1 workload
# (127 decode forwards), from two single-kernel ncu captures of the same call with fewer ids:
# `bench.py --case decode --new 24` (23 forwards) 102,231,552 B and `--new 48` (47 forwards)
# 121,998,592 B.  The first forward reads the weights from DRAM (ncu flushes the caches before the
# kernel, as the bench flushes L2 before each call); every later one adds (121,998,592 - 102,231,552)
# / 24 = 823,627 B.  127 forwards: 102,231,552 + 104 x 823,627 = 187,888,760 B.
DECODE_TRAFFIC_PER_LAUNCH = {("config1 petitgpt b1 p64 n128", "decode1"): 187_888_760}
# sm__pipe_tensor_cycles_active (% of peak, active cycles) of the decode-step GEMMs of config 5, one
# single-kernel ncu --set full capture each on `bench.py --case batched --seqs 128 --prompt 8 --new 3`
# (the first decode step's launch; mma.sync.m16n8k16 tiles): the share of the tensor pipe they keep busy.
BATCHED_TENSOR_PIPE = {"source": "ncu single-kernel captures: the mma.sync GEMMs and attention on a 128-row decode "
                                 "step; the tcgen05 lm_head (the default) on a 128-row forward of "
                                 "`bench.py --case batched --seqs 256 --prompt 8 --new 3`", "unit": "% of peak",
                       "lwe_gemm_qkv<2,4>": 11.9, "lwe_gemm_w13<2,1>": 20.9, "lwe_gemm_resid<2,4>": 5.0,
                       "lwe_lm_tc5<128,6>": 27.6, "lwe_attention<3,1>": 0.0}
# dram__bytes_read.sum + dram__bytes_write.sum of one cold gemv_q4_bulk_kernel launch on the lm_head
# shape (49152 x 576, M = 1), from an ncu capture of `bench.py --case gemv`: exactly the
# 17,694,720 bytes of nibbles and scales plus the activations.
GEMV_LM_TRAFFIC_PER_LAUNCH = 17_712_384


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


def decode_weight_bytes(cfg: dict) -> int:
    """Q4 weights (packed nibbles + fp32 group scales) plus fp32 norm gains of one forward."""
    return decode_algorithmic_bytes(cfg, 0, 1)


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
    written once; a decode step's attention reads the K/V rows of positions 0..pos of its own sequence;
    a prefill chunk reads each of its sequences' K/V rows once (as a flash-style kernel would: the
    re-reads of a causal prompt are not counted).  `chunks` = prefill forwards of the call."""
    d, ff, V, L = cfg["dModel"], cfg["dFf"], cfg["vocabSize"], cfg["nLayers"]
    kvd = cfg["nKvHeads"] * 64
    q4 = lambda r, c: r * c // 2 + r * (c // 32) * 4
    w = q4(V, d) + L * (q4(d + 2 * kvd, d) + q4(d, d) + 2 * q4(ff, d) + q4(d, ff)) + (2 * L + 1) * d * 4
    kv_row = 2 * L * kvd * 4
    total = chunks * w + 2 * nseq * plen * kv_row
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

WORKLOADS = {
    "decode": dict(model="petitgpt", seed=0, prompt=64, new=128, workload="config1 petitgpt b1 p64 n128",
                   metric="batch-1 Q4 decode tok/s (PetitGPT shape, 64-token prompt, 128 new tokens)",
                   model_text="PetitGPT-shaped Q4 (30L d576 9/3 ff1536 V32000)"),
    "gpt2": dict(model="gpt2", seed=2, prompt=128, new=256, workload="config3 gpt2 b1 p128 n256 argmaxGpt2",
                 metric="batch-1 Q4 decode tok/s (GPT-2 124M shape, 128-token prompt, 256 new tokens)",
                 model_text="GPT-2-shaped Q4 (12L d768 12 heads ff3072 V50257, LayerNorm, GELU, wpe)"),
    "spec4": dict(model="smollm2-360m", seed=3, prompt=512, new=256, spec_k=4, copy_spans=True,
                  workload="config4 smollm2-360m p512 n256 prompt-lookup k4 n3",
                  metric="batch-1 Q4 decode tok/s with prompt-lookup speculation (SmolLM2-360M shape, k=4)",
                  model_text="SmolLM2-360M-shaped Q4 (32L d960 15/5 ff2560 V49152)"),
    "spec8": dict(model="smollm2-360m", seed=3, prompt=512, new=256, spec_k=8, copy_spans=True,
                  workload="config4 smollm2-360m p512 n256 prompt-lookup k8 n3",
                  metric="batch-1 Q4 decode tok/s with prompt-lookup speculation (SmolLM2-360M shape, k=8)",
                  model_text="SmolLM2-360M-shaped Q4 (32L d960 15/5 ff2560 V49152)"),
}


def run_batched_leg(torch, P, local: int, rank: int, ws: int, dist, steps: int, warmup: int, cpu: bool):
    """BASELINE config 5 on this rank's GPU: 256 independent sequences (this rank's partition of the
    global set: sequence ids rank*256 ..), 128-token seeded prompts, 256 greedy new tokens, one
    mllm_generate_batch call per step.  Returns the sub-object for the JSON line (rank 0)."""
    B = BATCHED
    cfg = P.CONFIGS[B["model"]]
    data = P.synthetic_pgw(B["model"], B["seed"], cache_dir=CACHE)
    nseq, plen, nnew = B["nseq"], B["plen"], B["nnew"]
    seqs = [P.seeded_prompt(plen, cfg["vocabSize"], sd) for sd in batched_sequence_seeds(rank, nseq)]
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
    ev_ms, wall_ms = max_over_ranks(dist, [ev_ms, wall_ms], f"cuda:{local}")
    hbm, _, peak_kind = peaks()
    alg = batched_algorithmic_bytes(cfg, nseq, plen, nnew, chunks)
    ms = ev_ms / steps
    achieved = alg / (ms / 1e3) / 1e9
    out = {
        "metric": "replicated multi-sequence decode aggregate tok/s (SmolLM2-135M shape, 256 seqs/GPU, "
                  "128-token prompts, 256 new tokens)",
        "value": aggregate_rate(nseq * nnew, steps, ws, ev_ms), "unit": "tok/s", "n_gpus": ws, "steps": steps,
        "warmup": warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "config": {"workload": "config5 smollm2-135m 256 seqs/GPU p128 n256", "sequences_per_gpu": nseq,
                   "partition": "sequence ids rank*256 .. rank*256+255", "inputs": "larger than L2 (4.5 GB KV)",
                   "timing": "CUDA events around one mllm_generate_batch call (its 128 KB prompt upload and "
                             "256 KB id download included)"},
        "prefill_ms": float(np.mean(pre_ms)), "decode_tok_s_per_gpu": nseq * (nnew - 1) / ((np.mean(dev_ms) - np.mean(pre_ms)) / 1e3),
        "e2e": {"value": aggregate_rate(nseq * nnew, steps, ws, wall_ms), "unit": "tok/s",
                "h2d_bytes_per_step": nseq * plen * 4 + (3 * nseq * plen + 2 * nseq) * 4 + nseq * 4,
                "d2h_bytes_per_step": nseq * nnew * 4 + nseq * 4 + 17 * 4},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": peak_kind, "traffic": None, "kernel": "whole call: token-batch GEMMs (lwe_gemm_resid, _w13, _qkv, "
                     "_lm_wide: about 65 % of a decode step) and attention over the fp32 KV cache (lwe_attention, "
                     "about 34 %)", "algorithmic_bytes_per_step": alg},
        "tensor_pipe": BATCHED_TENSOR_PIPE,
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


def replica_prompt_seed(seed: int, rank: int) -> int:
    """Prompt seed of one batch-1 replica: every rank decodes its own sequence."""
    return seed + rank


def batched_sequence_seeds(rank: int, nseq: int) -> list:
    """Prompt seeds of this rank's partition of the config-5 sequence set (ids rank*nseq .. +nseq-1)."""
    return [4000 + rank * nseq + i for i in range(nseq)]


def max_over_ranks(dist, values, device) -> list:
    """Element-wise max of this rank's timings (ms) over all ranks; every rank receives the result.
    One all-reduce, the same on every rank. Without a process group the values come back unchanged."""
    if not dist:
        return [float(v) for v in values]
    import torch
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.cpu()]


def aggregate_rate(units_per_rank_step: int, steps: int, ws: int, max_ms: float) -> float:
    """Whole-job rate: the units all ranks processed over the max-over-ranks time, per second."""
    return units_per_rank_step * steps * ws / (max_ms / 1e3)


def config_of(W: dict, ws: int) -> dict:
    """The workload's `config` dict, identical in both arms (descriptive notes live outside it)."""
    return {"workload": W["workload"], "model": W["model_text"], "global_batch": ws,
            "seq_len": W["prompt"] + W["new"], "parallelism": "replicas"}


def run_reference(args):
    """--impl reference: the CPU restatement of the reference path (oracle/: engine/infer.js), all host
    threads, rank 0 only, on the default workload (config 1).  Every step is the whole workload: the
    64-token prefill and all 127 decode steps, greedy, as engine/infer.js:603-646 runs them."""
    ws, rank, _ = dist_setup()
    if rank != 0:
        return
    P = pkg()
    W = WORKLOADS["decode"]
    cfg = P.CONFIGS[W["model"]]
    data = P.synthetic_pgw(W["model"], W["seed"], cache_dir=CACHE)
    prompt = P.seeded_prompt(W["prompt"], cfg["vocabSize"], replica_prompt_seed(W["seed"], 0))
    threads = os.cpu_count() or 1
    from oracle.oracle import OracleModel
    om = OracleModel(data, threads=threads)
    for _ in range(args.warmup):
        om.generate(prompt, W["new"], eos=-1)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        r = om.generate(prompt, W["new"], eos=-1)
        times.append(time.perf_counter() - t0)
        assert len(r["generatedIds"]) == W["new"]
    wall = sum(times)
    v = W["new"] * args.steps / wall
    line = {
        "impl": "reference", "metric": W["metric"],
        "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": wall / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f64-accumulate/f32-store", "data": DATA_TEXT,
        "config": config_of(W, ws),  # the CUDA arm's dict at the same N (same_config)
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"every step the whole workload of one replica: {W['prompt']}-token prefill + "
                                   f"{W['new'] - 1} greedy decode steps (oracle/, the C restatement of "
                                   f"engine/infer.js; {threads} threads inside each forward; the host's cores "
                                   f"serve all {ws} replicas in turn at this rate)"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


GEMV_SHAPES = [(576, 576), (192, 576), (1536, 576), (576, 1536), (960, 960), (2560, 960), (960, 2560), (49152, 576)]


def gemv_points(torch, P, steps: int, shapes=GEMV_SHAPES, ms=(1, 5, 9, 16), modes=("hot", "cold")):
    """BASELINE config 2 points: isolated Q4 GEMV / skinny GEMM.  For every point both entry points are
    timed over a CUDA graph of back-to-back launches: `gemv` = mllm_gemv_q4 (CUDA-core, tensor-core or
    bulk-staged tensor-core kernel, picked per shape) and `gemm` = mllm_gemm_q4 (the token-batch
    tensor-core GEMM); hot = one weight matrix reused, cold = a rotating set of copies larger than L2.
    GB/s counts packed nibbles + scales (out*in/2 + out*in/32*4 bytes) per launch.  Returns (points,
    kernel launches)."""
    rng = np.random.default_rng(1)
    st = torch.cuda.Stream()
    rows, launches, reps = [], 0, 50
    for (R, C) in shapes:
        w = (rng.standard_normal((R, C), dtype=np.float32) * np.float32(0.02))
        packed, scales = P.quant_q4(w)
        bytes_w = packed.nbytes + scales.nbytes
        ncopy = max(1, -(-2 * L2_BYTES // bytes_w))
        pk = torch.from_numpy(np.ascontiguousarray(packed).reshape(-1)).cuda()
        sc = torch.from_numpy(np.ascontiguousarray(scales).reshape(-1)).cuda()
        pks = pk.repeat(ncopy).view(ncopy, -1)
        scs = sc.repeat(ncopy).view(ncopy, -1)
        for M in ms:
            x = torch.from_numpy(rng.standard_normal((M, C), dtype=np.float32)).cuda()
            y = torch.empty((M, R), device="cuda")
            point = {"shape": f"{R}x{C}", "M": M, "weight_bytes": bytes_w}
            for path, fn in (("gemv", P.gemv_q4_device), ("gemm", P.gemm_q4_device)):
                for mode in modes:
                    n = reps if mode == "hot" else min(ncopy, 4096)
                    idx = [0] * n if mode == "hot" else list(range(n))
                    with torch.cuda.stream(st):
                        for i in range(3):  # warm-up (allocates the GEMM workspace before capture)
                            fn(pks[0].data_ptr(), scs[0].data_ptr(), x.data_ptr(), y.data_ptr(), R, C, M, st.cuda_stream)
                    st.synchronize()
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=st):
                        for i in idx:
                            fn(pks[i].data_ptr(), scs[i].data_ptr(), x.data_ptr(), y.data_ptr(), R, C, M,
                               torch.cuda.current_stream().cuda_stream)
                    g.replay()
                    torch.cuda.synchronize()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    for _ in range(steps):
                        g.replay()
                    e1.record()
                    e1.synchronize()
                    us = e0.elapsed_time(e1) * 1e3 / (steps * n)
                    launches += steps * n * (1 if path == "gemv" else 2)
                    point[f"{path}_{mode}_us"] = us
                    point[f"{path}_{mode}_gbs"] = bytes_w / (us * 1e-6) / 1e9
                    del g
            if "cold" in modes:
                point["best_cold_gbs"] = max(point["gemv_cold_gbs"], point["gemm_cold_gbs"])
            if "hot" in modes:
                point["best_hot_gbs"] = max(point["gemv_hot_gbs"], point["gemm_hot_gbs"])
            rows.append(point)
        del pks, scs
    return rows, launches


def gemv_dense_points(torch, P, steps: int, R: int = 49152, C: int = 576, ms=(1, 16)):
    """mllm_gemv (f32 / f16 / bf16 / q8 storage, engine/infer.js:10-86) on the lm_head shape, cold L2
    (rotating copies larger than 2x L2, a CUDA graph of back-to-back launches).  GB/s counts the stored
    weight bytes (+ the q8 row scales) per launch.  Returns (points, kernel launches)."""
    rng = np.random.default_rng(1)
    st = torch.cuda.Stream()
    out, launches = [], 0
    w = rng.standard_normal((R, C), dtype=np.float32) * np.float32(0.02)
    for dt, esize in (("f32", 4), ("f16", 2), ("bf16", 2), ("q8", 1)):
        nbytes = R * C * esize + (R * 4 if dt == "q8" else 0)
        ncopy = max(1, -(-2 * L2_BYTES // nbytes))
        wt = torch.empty((ncopy, R * C * esize), dtype=torch.uint8, device="cuda")
        wt.random_(0, 256)
        if dt in ("f16", "bf16"):  # finite 16-bit words (the top bits of N(0, 0.02) values)
            wt.view(torch.int16).copy_(torch.from_numpy(w.astype(np.float16).view(np.int16)).cuda().reshape(-1))
        elif dt == "f32":
            wt.view(torch.float32).copy_(torch.from_numpy(w).cuda().reshape(-1))
        sc = torch.full((R,), 1e-3, device="cuda")
        for M in ms:
            x = torch.from_numpy(rng.standard_normal((M, C), dtype=np.float32)).cuda()
            y = torch.empty((M, R), device="cuda")
            n = min(ncopy, 4096)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                for i in range(n):
                    P.gemv_device(dt, wt[i].data_ptr(), sc.data_ptr(), x.data_ptr(), y.data_ptr(), R, C, M,
                                  torch.cuda.current_stream().cuda_stream)
            g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                g.replay()
            e1.record()
            e1.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (steps * n)
            launches += steps * n + n
            out.append({"dtype": dt, "shape": f"{R}x{C}", "M": M, "weight_bytes": nbytes, "cold_us": us,
                        "cold_gbs": nbytes / (us * 1e-6) / 1e9})
            del g
        del wt
    return out, launches


def gemv_e2e(torch, P, steps: int):
    """The headline GEMV point (lm_head 49152x576, M = 1) through the C ABI with host buffers: every
    step copies x from pinned host memory, runs mllm_gemv_q4 and reads y back; events around it."""
    R, C = 49152, 576
    rng = np.random.default_rng(1)
    packed, scales = P.quant_q4(rng.standard_normal((R, C), dtype=np.float32) * np.float32(0.02))
    pk = torch.from_numpy(np.ascontiguousarray(packed).reshape(-1)).cuda()
    sc = torch.from_numpy(np.ascontiguousarray(scales).reshape(-1)).cuda()
    hx = torch.from_numpy(rng.standard_normal((1, C), dtype=np.float32)).pin_memory()
    hy = torch.empty((1, R), dtype=torch.float32).pin_memory()
    x = torch.empty((1, C), device="cuda")
    y = torch.empty((1, R), device="cuda")
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")
    st = torch.cuda.Stream()
    total = 0.0
    for i in range(steps + 3):
        with torch.cuda.stream(st):
            flush.fill_(1.0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            x.copy_(hx, non_blocking=True)
            P.gemv_q4_device(pk.data_ptr(), sc.data_ptr(), x.data_ptr(), y.data_ptr(), R, C, 1, st.cuda_stream)
            hy.copy_(y, non_blocking=True)
            e1.record(st)
        e1.synchronize()
        if i >= 3:
            total += e0.elapsed_time(e1)
    us = total * 1e3 / steps
    return (packed.nbytes + scales.nbytes) / (us * 1e-6) / 1e9, C * 4, R * 4


def cpu_baseline_gemv(P, threads: int):
    """Oracle gemvQ4 (engine/infer.js:88-116, f64 sums) on the headline shape, all host threads."""
    from oracle.oracle import gemv_q4
    R, C = 49152, 576
    rng = np.random.default_rng(1)
    packed, scales = P.quant_q4(rng.standard_normal((R, C), dtype=np.float32) * np.float32(0.02))
    x = rng.standard_normal(C, dtype=np.float32)
    gemv_q4(packed, scales, x, threads=threads)
    t0 = time.perf_counter()
    n = 0
    while time.perf_counter() - t0 < 1.0:
        gemv_q4(packed, scales, x, threads=threads)
        n += 1
    dt = (time.perf_counter() - t0) / n
    return (packed.nbytes + scales.nbytes) / dt / 1e9, n


def gemv_line(torch, P, steps: int, full: bool, cpu: bool) -> dict:
    """Config 2 as a JSON object: the headline point (lm_head shape, M = 1, cold L2) with its roofline,
    e2e and CPU baseline, plus every shape x M point (cold; hot too when `full`)."""
    hbm, _, peak_kind = peaks()
    rows, launches = gemv_points(torch, P, steps, modes=("hot", "cold") if full else ("cold",))
    head = next(r for r in rows if r["shape"] == "49152x576" and r["M"] == 1)
    e2e, h2d, d2h = gemv_e2e(torch, P, max(steps, 3))
    out = {
        "metric": "Q4 g32 GEMV weight GB/s (lm_head 49152x576, M=1, cold L2)", "value": head["best_cold_gbs"],
        "unit": "GB/s", "n_gpus": 1, "steps": steps, "warmup": 3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q4xf32", "data": "synthetic (W ~ N(0,0.02) Q4 g32 seed 1, x ~ N(0,1))",
        "config": {"workload": "config2 gemv microbench", "shapes": [f"{r}x{c}" for r, c in GEMV_SHAPES],
                   "M": [1, 5, 9, 16], "timing": "CUDA graph of back-to-back launches, events around replays",
                   "cold": "rotating copies, total > 2x L2"},
        "e2e": {"value": e2e, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "hbm", "achieved": head["best_cold_gbs"], "peak": hbm, "unit": "GB/s",
                     "frac": head["best_cold_gbs"] / hbm, "peak_kind": peak_kind,
                     "traffic": GEMV_LM_TRAFFIC_PER_LAUNCH,
                     "kernel": "gemv_q4_bulk_kernel<1,2,2,2> (mllm_gemv_q4 on 49152x576, M=1; two CTAs per SM)"},
        "gpu_launches": launches, "points": rows,
    }
    dense, dl = gemv_dense_points(torch, P, steps)
    out["dense_points"] = dense  # the other PGW storage kinds (mllm_gemv), same shape, cold L2
    out["gpu_launches"] += dl
    if cpu:
        threads = os.cpu_count() or 1
        v, n = cpu_baseline_gemv(P, threads)
        out["cpu_baseline"] = {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                               "sample": f"oracle gemvQ4 (f64 sums) on 49152x576, M=1, {n} calls in 1 s"}
    return out


def run_gemv(args):
    """--workload gemv: config 2 alone (hot and cold), one JSON line."""
    import torch
    ws, rank, local = dist_setup()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    P = pkg()
    with ClockSampler(local) as clk:
        line = gemv_line(torch, P, args.steps, True, not args.no_cpu_baseline)
    line["warmup"] = args.warmup
    line["ms_per_step"] = None
    line["clocks"] = clk.summary()
    print(json.dumps(line), flush=True)


DATA_TEXT = "synthetic (seeded N(0,0.02) Q4 weights, seeded prompt ids; real checkpoints are LFS stubs)"


def measure_generate(torch, P, key: str, local: int, rank: int, ws: int, dist, steps: int, warmup: int,
                     cpu_threads: int, env: dict = None) -> dict:
    """One generate workload (configs 1, 3, 4) on this rank's GPU: `steps` timed generate calls after
    `warmup`, device path (prompt and ids resident in HBM) and e2e path (host buffers through
    mllm_generate), L2 flushed before each; max over ranks.  cpu_threads > 0 adds the oracle baseline on
    rank 0 at N = 1."""
    W = WORKLOADS[key]
    name, seed, n_prompt, n_new, spec_k = W["model"], W["seed"], W["prompt"], W["new"], W.get("spec_k", 0)
    cfg = P.CONFIGS[name]
    data = P.synthetic_pgw(name, seed, cache_dir=CACHE)
    if W.get("copy_spans"):
        prompt = P.copy_span_prompt(n_prompt, cfg["vocabSize"], replica_prompt_seed(seed, rank))
    else:
        prompt = P.seeded_prompt(n_prompt, cfg["vocabSize"], replica_prompt_seed(seed, rank))
    old_env = {k: os.environ.get(k) for k in (env or {})}
    os.environ.update(env or {})  # read by mllm_create only
    try:
        eng = P.CudaPetitGPT(data, device=local)
    finally:
        for k, v in old_env.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    stream = torch.cuda.Stream()
    eng.set_stream(stream.cuda_stream)
    d_ids = torch.from_numpy(prompt).to(f"cuda:{local}")
    d_out = torch.zeros(n_new + 16, dtype=torch.int32, device=f"cuda:{local}")
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=f"cuda:{local}")
    h_prompt = torch.from_numpy(prompt).pin_memory()
    h_out = torch.zeros(n_new + 16, dtype=torch.int32).pin_memory()
    launches = [0]
    spec_stats = []

    def step_device(k=spec_k):
        st = eng.generate_device(d_ids.data_ptr(), n_prompt, d_out.data_ptr(), n_new, -1, k, 3)
        assert st.n_generated == n_new, st.n_generated
        launches[0] += st.kernel_launches
        spec_stats.append((st.spec_hits, st.spec_tries, st.forwards))
        return st

    def step_e2e():
        import ctypes
        st = P.engine.Stats()
        eng._check(eng._lib.mllm_generate(eng._h, 0, ctypes.c_void_p(h_prompt.data_ptr()), n_prompt, n_new, -1, spec_k,
                                          3, ctypes.c_void_p(h_out.data_ptr()), ctypes.byref(st)))
        assert st.n_generated == n_new

    def timed(fn, k):
        """k steps, each bracketed by events on the launch stream, L2 flushed before each step."""
        total = 0.0
        dev_ms.clear()
        first_ms.clear()
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
                first_ms.append(st.ttft_ms)
        return total, list(dev_ms), list(first_ms)

    dev_ms, first_ms = [], []
    for _ in range(warmup):
        step_device()
        step_e2e()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    launches[0] = 0
    spec_stats.clear()
    with ClockSampler(local) as clk:
        t_dev, dev_v, first_v = timed(step_device, steps)
        torch.cuda.synchronize()
        t_e2e, _, _ = timed(step_e2e, steps)
    torch.cuda.synchronize()
    gpu_launches = launches[0]
    t_dev, t_e2e = max_over_ranks(dist, [t_dev, t_e2e], f"cuda:{local}")
    value = aggregate_rate(n_new, steps, ws, t_dev)
    e2e = aggregate_rate(n_new, steps, ws, t_e2e)
    ms_step = t_dev / steps
    hbm, _, peak_kind = peaks()
    alg = decode_algorithmic_bytes(cfg, n_prompt, n_new)
    w_bytes = decode_weight_bytes(cfg)
    kname = eng.decodeKernel
    if spec_k:  # the whole call is the unit: graph-replayed speculation iterations
        alg_launch, launch_ms = alg, ms_step
        traffic = None
    else:  # the persistent single-token launch: the decode forwards after the first id
        prefill = w_bytes + n_prompt * 2 * cfg["nLayers"] * cfg["nKvHeads"] * 64 * 4
        alg_launch = alg - prefill
        launch_ms = float(np.mean([t - f for t, f in zip(dev_v, first_v)])) if dev_v else ms_step
        traffic = DECODE_TRAFFIC_PER_LAUNCH.get((W["workload"], kname.split(":")[0]))
    achieved = alg_launch / (launch_ms / 1e3) / 1e9
    line = {
        "metric": W["metric"],
        "value": value, "unit": "tok/s", "n_gpus": ws, "steps": steps, "warmup": warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q4xf32",
        "data": DATA_TEXT,
        "config": config_of(W, ws),
        "notes": {"l2": (f"flushed (256 MB write) before every timed step; Q4 weights {w_bytes / 1e6:.0f} MB "
                         + ("fit in L2 within a step" if w_bytes < L2_BYTES else
                            "exceed L2, re-read from HBM every forward")),
                  "tokens_per_step": n_new, "launches_per_step": gpu_launches // max(steps, 1),
                  "path": (f"prefill as token-batch tensor-core forwards, then one CUDA-graph replay per "
                           f"speculation iteration (k_spec_prepare, {spec_k + 1}-row verify forward, k_spec_accept)"
                           if spec_k else
                           f"prefill as token-batch tensor-core forwards, then the {n_new - 1} decode steps in one "
                           f"persistent single-token kernel launch ({kname})")},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": n_prompt * 4, "d2h_bytes_per_step": n_new * 4 + 68},
        "gpu_launches": gpu_launches,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": peak_kind, "traffic": traffic,
                     "limiter": ("latency: the weights stay L2-resident between tokens (DRAM traffic "
                                 f"{traffic / alg_launch:.1%} of the algorithmic bytes), so the per-layer chain of "
                                 "stage exchanges sets the time" if traffic else
                                 "latency of the per-token chain of stages (see the profiles)"),
                     "kernel": ("whole generate call (token-batch prefill + graph-replayed speculation iterations)"
                                if spec_k else f"{kname}: the {n_new - 1} decode forwards after the first id"),
                     "algorithmic_bytes_per_launch": alg_launch,
                     "launch_ms_device_timer": launch_ms,
                     "traffic_source": ("two single-kernel ncu captures (23 and 47 forwards) scaled to "
                                        f"{n_new - 1} forwards" if traffic else None)},
        "clocks": clk.summary(),
    }
    if spec_k:
        hits = sum(h for h, _, _ in spec_stats[:steps]) / steps
        tries = sum(t for _, t, _ in spec_stats[:steps]) / steps
        fw = sum(f for _, _, f in spec_stats[:steps]) / steps
        line["speculation"] = {"spec_k": spec_k, "ngram": 3, "spec_hits": hits, "spec_tries": tries,
                               "acceptance_rate": hits / max(tries * spec_k, 1), "accepted_per_try": hits / max(tries, 1),
                               "forwards_per_call": fw, "tokens_per_forward": n_new / max(fw, 1)}
        # the same model and prompt without speculation, for the speed-up (same timing, same flush)
        t_g, _, _ = timed(lambda: step_device(0), max(2, min(steps, 3)))
        t_g = max_over_ranks(dist, [t_g], f"cuda:{local}")[0]
        greedy = n_new * max(2, min(steps, 3)) / (t_g / 1e3)
        line["speculation"]["greedy_tok_s"] = greedy
        line["speculation"]["speedup_vs_greedy"] = (value / ws) / greedy
    if rank == 0 and ws == 1 and cpu_threads > 0:
        sample = 4
        v, pre, per = cpu_baseline_decode(data, prompt, n_new, cpu_threads, sample)
        line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": cpu_threads, "kind": "port",
                                "sample": f"oracle (C restatement of engine/infer.js), {cpu_threads} thread(s): "
                                          f"{n_prompt}-token prefill ({pre:.2f} s) + {sample} greedy decode steps "
                                          f"({per*1e3:.0f} ms/token), extrapolated to {n_new - 1} decode steps"}
    eng.destroy()
    return line


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
    cpu = not args.no_cpu_baseline
    line = measure_generate(torch, P, args.workload, local, rank, ws, dist, args.steps, args.warmup, 1 if cpu else 0)
    if args.workload == "decode" and not args.no_batched:
        line["batched"] = run_batched_leg(torch, P, local, rank, ws, dist, args.batched_steps, 1, cpu)
    if args.workload == "decode" and not args.no_extra:
        threads = os.cpu_count() or 1
        ls, lw = args.leg_steps, 2
        # config 1 on the cluster decode kernel (one 16-CTA cluster per kv head; opt-in in the engine)
        line["decode_cluster"] = measure_generate(torch, P, "decode", local, rank, ws, dist, ls, lw, 0,
                                                  env={"MLLM_CLUSTER_DECODE": "1"})
        line["gpt2"] = measure_generate(torch, P, "gpt2", local, rank, ws, dist, ls, lw, threads if cpu else 0)
        line["spec4"] = measure_generate(torch, P, "spec4", local, rank, ws, dist, ls, lw, 0)
        line["spec8"] = measure_generate(torch, P, "spec8", local, rank, ws, dist, ls, lw, 0)
        if cpu and rank == 0 and ws == 1:
            W = WORKLOADS["spec4"]
            data = P.synthetic_pgw(W["model"], W["seed"], cache_dir=CACHE)
            prompt = P.copy_span_prompt(W["prompt"], P.CONFIGS[W["model"]]["vocabSize"], W["seed"])
            v, pre, per = cpu_baseline_decode(data, prompt, W["new"], threads, 2)
            cb = {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                  "sample": f"oracle greedy (no speculation), {threads} threads: {W['prompt']}-token prefill "
                            f"({pre:.2f} s) + 2 decode steps ({per*1e3:.0f} ms/token), extrapolated to "
                            f"{W['new'] - 1} decode steps"}
            line["spec4"]["cpu_baseline"] = cb
            line["spec8"]["cpu_baseline"] = cb
        if rank == 0:
            line["gemv"] = gemv_line(torch, P, 3, False, cpu)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


TIMELINE_STAGES = ["x2 wait + residual + act", "1/RMS", "q/k/v rows (units + epilogue)", "q/k/v push",
                   "q/k/v wait", "RoPE + q/k", "K/V staging wait + cache row", "attention (scores, softmax, v)",
                   "partial push", "partials wait", "merge -> proj activation", "proj columns (units + epilogue)",
                   "x1 publish (global + forward)", "x1 wait", "x1 residual + act + 1/RMS",
                   "w1/w3 rows (units)", "SiLU(u) v", "w2 columns (units + epilogue)", "reduce-scatter push",
                   "reduce-scatter wait", "x2 publish (sum + global + forward)"]


def run_timeline(args):
    """Stage timeline of the cluster decode kernel (see run_case); the stamps are globaltimer values of
    thread 0 of every CTA, each stage the difference of max-over-CTA stamps."""
    import ctypes
    P = pkg()
    lib = os.path.join(ROOT, "microllm-lab_b200", "libmllm_cuda_timeline.so")
    L = P.engine.load_library(lib)
    if not os.path.samefile(L._name, lib):
        raise RuntimeError("the timeline library must be the first libmllm loaded in the process")
    os.environ["MLLM_CLUSTER_DECODE"] = "1"
    W = WORKLOADS["decode"]
    cfg = P.CONFIGS[W["model"]]
    data = P.synthetic_pgw(W["model"], W["seed"], cache_dir=CACHE)
    prompt = P.seeded_prompt(W["prompt"], cfg["vocabSize"], W["seed"])
    eng = P.CudaPetitGPT(data)
    if "cdec" not in eng.decodeKernel:
        raise RuntimeError(f"cluster decode is not available for this model: {eng.decodeKernel}")
    nc = int(eng.decodeKernel.split(":")[1].split()[0])
    L.mllm_timeline_config.argtypes = [ctypes.c_int]
    L.mllm_timeline_dump.argtypes = [ctypes.c_void_p, ctypes.c_int]
    if L.mllm_timeline_config(args.forward):
        raise RuntimeError("mllm_timeline_config failed")
    nnew = max(args.new or 24, args.forward + 2)
    g = eng.generate(prompt, maxNewTokens=nnew, eosId=-1)
    st = np.zeros((16 * nc, 1024), np.uint64)
    if L.mllm_timeline_dump(st.ctypes.data, 16 * nc):
        raise RuntimeError("mllm_timeline_dump failed")
    eng.destroy()
    mx = st.astype(np.int64).max(axis=0)
    nl, per = cfg["nLayers"], 24
    rows = []
    for k in range(1, len(TIMELINE_STAGES) + 1):
        d = [(mx[l * per + k] - mx[l * per + k - 1]) / 1e3 for l in range(nl)]
        rows.append({"stage": TIMELINE_STAGES[k - 1], "us_mean": round(float(np.mean(d)), 3),
                     "us_layer15": round(float(d[min(15, nl - 1)]), 3)})
    layer_us = [(mx[(l + 1) * per] - mx[l * per]) / 1e3 for l in range(nl - 1)]
    tail = {"x2 wait + final norm": (mx[1001] - mx[1000]) / 1e3, "lm_head rows": (mx[1002] - mx[1001]) / 1e3,
            "stream end + argmax": (mx[1003] - mx[1002]) / 1e3, "candidate exchange": (mx[1004] - mx[1003]) / 1e3}
    print(json.dumps({"case": "timeline", "kernel": f"cdec_kernel, {nc} clusters of 16 CTAs",
                      "forward": args.forward, "position": W["prompt"] + args.forward,
                      "layer_us_mean": round(float(np.mean(layer_us)), 3),
                      "token_us": round((mx[1004] - mx[0]) / 1e3, 2), "stages": rows,
                      "tail_us": {k: round(float(v), 3) for k, v in tail.items()},
                      "deviceMs": g["deviceMs"], "new": nnew}, indent=1))


def run_case(args):
    """One small, untimed run of a path, sized for a profiler capture (``--case``; prints one summary line).

    decode:  a BASELINE config-1 generate call (PetitGPT shape, seed 0, 64-token prompt) with --new ids;
    timeline: the same call on the cluster decode kernel from libmllm_cuda_timeline.so (built by
             ``build.py --timeline``), printing the per-stage times of forward --forward: per layer and
             stage the max over CTAs of the stage's closing stamp minus the previous one, averaged over
             the layers, and the lm_head tail;
    batched: config 5 (SmolLM2-135M shape) with --seqs sequences of --prompt-token prompts (default 128)
             and --new ids;
    spec:    config 4 (SmolLM2-360M shape, 512-token copy-span prompt) with --new ids at k = --k;
    gemv:    one cold mllm_gemv_q4 on the lm_head shape (49152 x 576, M = 1);
    gemm:    two mllm_gemm_q4 calls (tcgen05 tiles) on --rows x --cols with --seqs activation rows."""
    import torch
    if args.case == "timeline":
        run_timeline(args)
        return
    P = pkg()
    if args.case == "gemm":  # one mllm_gemm_q4 (tcgen05 tiles) on --rows x --cols with --seqs activation rows
        rows, cols, m = args.rows, args.cols, args.seqs
        rng = np.random.default_rng(1)
        packed, scales = P.quant_q4(rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))
        pk = torch.from_numpy(np.ascontiguousarray(packed).reshape(-1)).cuda()
        sc = torch.from_numpy(np.ascontiguousarray(scales).reshape(-1)).cuda()
        x = torch.from_numpy(rng.standard_normal((m, cols), dtype=np.float32)).cuda()
        y = torch.empty((m, rows), device="cuda")
        for _ in range(2):
            P.gemm_q4_device(pk.data_ptr(), sc.data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, m)
        torch.cuda.synchronize()
        print(json.dumps({"case": "gemm", "rows": rows, "cols": cols, "m": m, "checksum": float(y.double().sum())}))
        return
    if args.case == "gemv":
        rows, cols = 49152, 576
        rng = np.random.default_rng(1)
        packed, scales = P.quant_q4(rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))
        pk = torch.from_numpy(np.ascontiguousarray(packed).reshape(-1)).cuda()
        sc = torch.from_numpy(np.ascontiguousarray(scales).reshape(-1)).cuda()
        x = torch.from_numpy(rng.standard_normal((1, cols), dtype=np.float32)).cuda()
        y = torch.empty((1, rows), device="cuda")
        P.gemv_q4_device(pk.data_ptr(), sc.data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, 1)
        torch.cuda.synchronize()
        print(json.dumps({"case": "gemv", "rows": rows, "cols": cols, "checksum": float(y.double().sum())}))
        return
    if args.case == "batched":
        B = BATCHED
        cfg = P.CONFIGS[B["model"]]
        data = P.synthetic_pgw(B["model"], B["seed"], cache_dir=CACHE)
        nnew, plen = args.new or 3, args.prompt or B["plen"]
        seqs = [P.seeded_prompt(plen, cfg["vocabSize"], sd) for sd in batched_sequence_seeds(0, args.seqs)]
        eng = P.CudaPetitGPT(data, max_slots=args.seqs, kv_len=plen + nnew)
        _, stats = eng.generateBatch(seqs, maxNewTokens=nnew, eosId=-1)
        print(json.dumps({"case": "batched", "seqs": args.seqs, "prompt": plen, "new": nnew, "stats": stats}))
        eng.destroy()
        return
    key = "spec4" if args.case == "spec" else "decode"
    W = WORKLOADS[key]
    cfg = P.CONFIGS[W["model"]]
    data = P.synthetic_pgw(W["model"], W["seed"], cache_dir=CACHE)
    if W.get("copy_spans"):
        prompt = P.copy_span_prompt(W["prompt"], cfg["vocabSize"], W["seed"])
    else:
        prompt = P.seeded_prompt(W["prompt"], cfg["vocabSize"], W["seed"])
    eng = P.CudaPetitGPT(data)
    nnew = args.new or 24
    g = eng.generate(prompt, maxNewTokens=nnew, eosId=-1, specK=args.k if args.case == "spec" else 0)
    print(json.dumps({"case": args.case, "kernel": eng.decodeKernel, "new": nnew, "deviceMs": g["deviceMs"],
                      "ids": g["generatedIds"][:8]}))
    eng.destroy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "gpt2", "spec4", "spec8", "gemv"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batched", action="store_true", help="skip the config-5 batched sub-object")
    ap.add_argument("--batched-steps", type=int, default=3)
    ap.add_argument("--leg-steps", type=int, default=3, help="timed steps of the config 3 and 4 sub-objects")
    ap.add_argument("--no-extra", action="store_true", help="only config 1 (and config 5 unless --no-batched)")
    ap.add_argument("--case", choices=["decode", "timeline", "batched", "spec", "gemv", "gemm"],
                    help="one small untimed run for a profiler capture (see run_case)")
    ap.add_argument("--new", type=int, default=0, help="--case: ids to generate")
    ap.add_argument("--seqs", type=int, default=128, help="--case batched: sequences")
    ap.add_argument("--prompt", type=int, default=0, help="--case batched: prompt tokens (0 = config 5's 128)")
    ap.add_argument("--k", type=int, default=4, help="--case spec: draft length")
    ap.add_argument("--forward", type=int, default=20, help="--case timeline: the stamped forward of the launch")
    ap.add_argument("--rows", type=int, default=1536, help="--case gemm: weight rows")
    ap.add_argument("--cols", type=int, default=576, help="--case gemm: columns (K)")
    args = ap.parse_args()
    if args.case:
        run_case(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload == "gemv":
        run_gemv(args)
    else:
        run_decode(args)


if __name__ == "__main__":
    main()
