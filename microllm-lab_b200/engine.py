"""Python host side of the B200 Q4 decode backend: ctypes over libmllm_cuda.so (include/mllm.h).

``CudaPetitGPT`` mirrors the engine surface MicroLLM lab's callers use (engine/worker.js:59-109,
149-159): the CPU ``PetitGPT`` of engine/infer.js:289-647 (``forwardPrompt``, ``forwardDecode``,
``resetCache``, ``cacheLen``, ``cfg``, ``kind``, ``generate``) and the GPU-engine extras of
engine/webgpu.js:867-1297 (``init``, ``destroy``, ``bytesAllocated``, ``mode``, ``ready``,
``specHits``/``specTries`` in the result).  Method names keep the reference's camelCase so that
code written against it reads the same.

There is no CPU fallback: if the shared library or a CUDA device is missing, construction raises.
"""
from __future__ import annotations

import ctypes
import os
import time

import numpy as np

from .pgw import Bundle, parse_pgw

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmllm_cuda.so")
SPECIAL = {"PAD": 0, "UNK": 1, "BOS": 2, "EOS": 3, "SYSTEM": 4, "USER": 5, "ASSISTANT": 6}  # engine/tokenizer.js:188-196
STOP_NAMES = {0: "eos", 1: "max_new_tokens", 2: "context_limit"}
PHASE_NAMES = {0: "prefill", 1: "decode", 2: "spec"}  # onToken phases (engine/infer.js:615,630; webgpu.js:1253,1265)
TOKEN_FN = ctypes.CFUNCTYPE(None, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p)

EXPORTS = ["mllm_create", "mllm_destroy", "mllm_last_error", "mllm_config", "mllm_set_stream", "mllm_bytes_allocated",
           "mllm_decode_kernel", "mllm_reset",
           "mllm_cache_len", "mllm_forward", "mllm_generate", "mllm_generate_stream", "mllm_generate_device",
           "mllm_generate_batch",
           "mllm_selftest_timeout",
           "mllm_gemv_q4", "mllm_gemv", "mllm_gemm_q4", "mllm_gemm_q4_noalloc"]


class MllmError(RuntimeError):
    """Raised for a non-zero mllm_status; mirrors the reference's ``throw new Error(message)``."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{message} (status {code})")
        self.code = code


class Stats(ctypes.Structure):
    _fields_ = [("n_generated", ctypes.c_int32), ("stop_reason", ctypes.c_int32), ("spec_hits", ctypes.c_int32),
                ("spec_tries", ctypes.c_int32), ("forwards", ctypes.c_int32), ("prompt_len", ctypes.c_int32),
                ("ttft_ms", ctypes.c_float), ("total_ms", ctypes.c_float), ("kernel_launches", ctypes.c_int32)]


class BatchStats(ctypes.Structure):
    _fields_ = [("n_seq", ctypes.c_int32), ("total_generated", ctypes.c_int32), ("steps", ctypes.c_int32),
                ("prefill_forwards", ctypes.c_int32), ("prefill_ms", ctypes.c_float), ("total_ms", ctypes.c_float),
                ("kernel_launches", ctypes.c_int32)]


_LIB = None


def load_library(path: str = LIB_PATH):
    """Load libmllm_cuda.so and declare its C signatures.  Raises if the library is absent."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise OSError(f"{path} is missing: build it with `python microllm-lab_b200/build.py`")
    L = ctypes.CDLL(path)
    P, I, Z = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
    L.mllm_create.argtypes = [I, P, Z, I, I, ctypes.POINTER(P)]
    L.mllm_destroy.argtypes = [P]
    L.mllm_destroy.restype = None
    L.mllm_last_error.argtypes = [P]
    L.mllm_last_error.restype = ctypes.c_char_p
    L.mllm_config.argtypes = [P, P]
    L.mllm_bytes_allocated.argtypes = [P]
    L.mllm_bytes_allocated.restype = Z
    L.mllm_decode_kernel.argtypes = [P]
    L.mllm_decode_kernel.restype = ctypes.c_char_p
    L.mllm_reset.argtypes = [P, I]
    L.mllm_cache_len.argtypes = [P, I]
    L.mllm_forward.argtypes = [P, I, P, I, I, I, P, P]
    L.mllm_generate.argtypes = [P, I, P, I, I, ctypes.c_int32, I, I, P, ctypes.POINTER(Stats)]
    L.mllm_generate_device.argtypes = [P, I, P, I, I, ctypes.c_int32, I, I, P, ctypes.POINTER(Stats)]
    L.mllm_generate_stream.argtypes = [P, I, P, I, I, ctypes.c_int32, I, I, P, ctypes.POINTER(Stats), TOKEN_FN, P]
    L.mllm_generate_batch.argtypes = [P, I, P, P, I, ctypes.c_int32, P, P, P, ctypes.POINTER(BatchStats)]
    L.mllm_gemv_q4.argtypes = [P, P, P, P, I, I, I, P]
    L.mllm_gemv.argtypes = [I, P, P, P, P, I, I, I, P]
    L.mllm_gemm_q4.argtypes = [P, P, P, P, I, I, I, P]
    L.mllm_gemm_q4_noalloc.argtypes = [P, P, P, P, I, I, I, P]
    L.mllm_selftest_timeout.argtypes = [P, I]
    L.mllm_set_stream.argtypes = [P, P]
    _LIB = L
    return L


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def gemv_q4_device(packed_ptr: int, scales_ptr: int, x_ptr: int, y_ptr: int, rows: int, cols: int, n_act: int,
                   stream: int = 0) -> None:
    """Q4 GEMV on device pointers (mllm_gemv_q4): y[n_act][rows] = x[n_act][cols] . W^T."""
    rc = load_library().mllm_gemv_q4(packed_ptr, scales_ptr, x_ptr, y_ptr, rows, cols, n_act, stream or None)
    if rc:
        raise MllmError(rc, "mllm_gemv_q4 rejected its arguments")


DTYPES = {"f32": 0, "f16": 1, "bf16": 2, "q8": 3, "q4": 4}  # engine/weights.js:3 (mllm_dtype)


def gemv_device(dtype: str, w_ptr: int, scales_ptr: int, x_ptr: int, y_ptr: int, rows: int, cols: int, n_act: int,
                stream: int = 0) -> None:
    """GEMV for the f32 / f16 / bf16 / q8 storage kinds on device pointers (mllm_gemv):
    y[n_act][rows] = x[n_act][cols] . W^T (q8: times the row scales)."""
    rc = load_library().mllm_gemv(DTYPES[dtype], w_ptr, scales_ptr or None, x_ptr, y_ptr, rows, cols, n_act,
                                  stream or None)
    if rc:
        raise MllmError(rc, "mllm_gemv rejected its arguments")


def gemm_q4_device(packed_ptr: int, scales_ptr: int, x_ptr: int, y_ptr: int, rows: int, cols: int, n_act: int,
                   stream: int = 0) -> None:
    """Tensor-core Q4 GEMM on device pointers (mllm_gemm_q4): y[n_act][rows] = x[n_act][cols] . W^T."""
    rc = load_library().mllm_gemm_q4(packed_ptr, scales_ptr, x_ptr, y_ptr, rows, cols, n_act, stream or None)
    if rc:
        raise MllmError(rc, "mllm_gemm_q4 failed")


class CudaPetitGPT:
    """B200 engine with the PetitGPT surface (engine/infer.js:289-647, engine/webgpu.js:867-1297)."""

    def __init__(self, bundle, device: int = 0, max_slots: int = 1, kv_len: int = 0, slot: int = 0):
        if isinstance(bundle, Bundle):
            data = bundle.buffer
        else:
            data = bytes(bundle)
            bundle = parse_pgw(data)
        self.bundle = bundle
        self.cfg = dict(bundle.cfg)
        self.kind = bundle.kind
        self.device = device
        self.slot = slot
        self._lib = load_library()
        h = ctypes.c_void_p()
        buf = np.frombuffer(data, np.uint8)
        rc = self._lib.mllm_create(device, _ptr(buf), buf.nbytes, max_slots, kv_len, ctypes.byref(h))
        if rc:
            raise MllmError(rc, self._lib.mllm_last_error(None).decode())
        self._h = h
        c = np.zeros(10, np.int32)
        self._lib.mllm_config(self._h, _ptr(c))
        self.maxTokensPerForward = int(c[9])
        self.kvLen = int(c[8])
        self.headDim = self.cfg["dModel"] // self.cfg["nHeads"]
        self.isGpt2 = self.cfg["arch"] == "gpt2"
        self.mode = "cuda-sm100a"
        self.ready = True

    # ---- lifecycle (engine/webgpu.js:892, 1284-1297)
    async def init(self):
        return self

    def destroy(self):
        if getattr(self, "_h", None):
            self._lib.mllm_destroy(self._h)
            self._h = None
        self.ready = False

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass

    def set_stream(self, stream_ptr: int):
        """Launch on the caller's cudaStream_t (0 = the handle's own stream)."""
        self._check(self._lib.mllm_set_stream(self._h, stream_ptr or None))

    @property
    def bytesAllocated(self) -> int:
        return int(self._lib.mllm_bytes_allocated(self._h))

    @property
    def decodeKernel(self) -> str:
        """The kernel that runs single-token decode on this handle."""
        return self._lib.mllm_decode_kernel(self._h).decode()

    def _check(self, rc: int):
        if rc:
            raise MllmError(rc, self._lib.mllm_last_error(self._h).decode())

    # ---- cache (engine/infer.js:348-358)
    def resetCache(self):
        self._check(self._lib.mllm_reset(self._h, self.slot))

    @property
    def cacheLen(self) -> int:
        return int(self._lib.mllm_cache_len(self._h, self.slot))

    # ---- forwards (engine/infer.js:553-601, engine/webgpu.js:1248)
    def forward(self, ids, pos0: int, logits_each: bool = False, want_logits: bool = True):
        """Forward over ``ids`` at positions pos0..; returns (logits, argmax) with logits [vocab] for
        the last row or [n][vocab] when logits_each."""
        ids = np.ascontiguousarray(ids, np.int32)
        n = len(ids)
        V = self.cfg["vocabSize"]
        rows = n if logits_each else 1
        logits = np.empty((rows, V), np.float32) if want_logits else None
        am = np.empty(rows, np.int32)
        self._check(self._lib.mllm_forward(self._h, self.slot, _ptr(ids), n, pos0, int(logits_each),
                                           _ptr(logits) if want_logits else None, _ptr(am)))
        if logits is not None and not logits_each:
            logits = logits[0]
        return logits, am

    def forwardPrompt(self, ids):
        """engine/infer.js:553-577 — resets the cache, returns the last position's logits."""
        self.resetCache()
        return self.forward(ids, 0)[0]

    def forwardDecode(self, tokenId: int):
        """engine/infer.js:579-601 — one token at position cacheLen."""
        return self.forward([int(tokenId)], self.cacheLen)[0]

    # ---- generation (engine/infer.js:603-646, engine/webgpu.js:1164-1282)
    def generate(self, ids, maxNewTokens: int = 64, eosId: int = SPECIAL["EOS"], onToken=None, specK: int = 0,
                 ngram: int = 3):
        """Greedy generation in one device launch.  ``specK > 0`` turns on prompt-lookup speculation
        (n-gram size ``ngram``), which runs on the device.  ``onToken(id, meta)`` is called for each id
        while the device is still generating (mllm_generate_stream: the kernels publish every id into
        mapped host memory as it is chosen), with phase "prefill" (and ``ms``, the host time since the
        call began) for the first id, "decode" for the others, and "spec" for accepted draft ids, as
        engine/infer.js:615,630 and engine/webgpu.js:1253,1265 report them."""
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.zeros(max(int(maxNewTokens), 1), np.int32)
        st = Stats()
        t0 = time.perf_counter()
        if onToken is None:
            self._check(self._lib.mllm_generate(self._h, self.slot, _ptr(ids), len(ids), int(maxNewTokens),
                                                int(eosId), int(specK), int(ngram), _ptr(out), ctypes.byref(st)))
        else:
            errors = []

            def cb(tok, index, phase, _user):
                if errors:
                    return
                meta = {"phase": PHASE_NAMES.get(int(phase), "decode")}
                if index == 0:
                    meta["ms"] = (time.perf_counter() - t0) * 1e3
                try:
                    onToken(int(tok), meta)
                except BaseException as ex:  # raised again once the call returns
                    errors.append(ex)

            fn = TOKEN_FN(cb)
            self._check(self._lib.mllm_generate_stream(self._h, self.slot, _ptr(ids), len(ids), int(maxNewTokens),
                                                       int(eosId), int(specK), int(ngram), _ptr(out), ctypes.byref(st),
                                                       fn, None))
            if errors:
                raise errors[0]
        wall = (time.perf_counter() - t0) * 1e3
        gen = out[:st.n_generated].tolist()
        return {
            "generatedIds": gen,
            "stopReason": STOP_NAMES.get(st.stop_reason, "max_new_tokens"),
            "ttftMs": float(st.ttft_ms),
            "totalMs": wall,
            "deviceMs": float(st.total_ms),
            "mode": self.mode,
            "specHits": int(st.spec_hits),
            "specTries": int(st.spec_tries),
            "forwards": int(st.forwards),
            "kernelLaunches": int(st.kernel_launches),
        }

    def generateBatch(self, seqs, maxNewTokens: int = 64, eosId: int = SPECIAL["EOS"]):
        """Replicated multi-sequence greedy decode (mllm_generate_batch): ``seqs`` is a list of prompts;
        sequence s runs on slot s.  Returns (results, stats) where results[s] is the dict
        ``generate`` would return for that prompt alone (generatedIds, stopReason) and stats holds the
        batch counters and device times."""
        seqs = [np.ascontiguousarray(q, np.int32) for q in seqs]
        n = len(seqs)
        offs = np.zeros(n + 1, np.int32)
        offs[1:] = np.cumsum([len(q) for q in seqs])
        flat = np.concatenate(seqs) if n else np.zeros(0, np.int32)
        flat = np.ascontiguousarray(flat, np.int32)
        out = np.zeros((n, max(int(maxNewTokens), 1)), np.int32)
        n_out = np.zeros(n, np.int32)
        stop = np.zeros(n, np.int32)
        st = BatchStats()
        t0 = time.perf_counter()
        self._check(self._lib.mllm_generate_batch(self._h, n, _ptr(flat), _ptr(offs), int(maxNewTokens), int(eosId),
                                                  _ptr(out), _ptr(n_out), _ptr(stop), ctypes.byref(st)))
        wall = (time.perf_counter() - t0) * 1e3
        res = [{"generatedIds": out[i, :n_out[i]].tolist(), "stopReason": STOP_NAMES.get(int(stop[i]), "max_new_tokens")}
               for i in range(n)]
        stats = {"nSeq": int(st.n_seq), "totalGenerated": int(st.total_generated), "steps": int(st.steps),
                 "prefillForwards": int(st.prefill_forwards), "prefillMs": float(st.prefill_ms),
                 "deviceMs": float(st.total_ms), "totalMs": wall, "kernelLaunches": int(st.kernel_launches)}
        return res, stats

    def selftest_timeout(self, wait_ms: int = 50) -> int:
        """Run the device wait-limit self-test; returns the mllm_status (MLLM_ERR_TIMEOUT = -6 expected)."""
        return int(self._lib.mllm_selftest_timeout(self._h, int(wait_ms)))

    def generate_device(self, d_ids: int, n: int, d_out: int, maxNewTokens: int, eosId: int = -1, specK: int = 0,
                        ngram: int = 3) -> Stats:
        """mllm_generate_device: prompt and output already in device memory (raw pointers)."""
        st = Stats()
        self._check(self._lib.mllm_generate_device(self._h, self.slot, d_ids, n, int(maxNewTokens), int(eosId),
                                                   int(specK), int(ngram), d_out, ctypes.byref(st)))
        return st
