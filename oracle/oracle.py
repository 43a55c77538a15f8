"""ctypes wrapper around liboracle.so, the C restatement of engine/infer.js.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
legs as the parity checker.  The CUDA product never imports it.

The PGW1 table reader here is deliberately independent of the product's parser; it restates
engine/weights.js:5-40 directly.
"""
from __future__ import annotations

import ctypes
import json
import os
import struct
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
STOP_NAMES = {0: "eos", 1: "max_new_tokens", 2: "context_limit"}


def build() -> str:
    so = os.path.join(_HERE, "liboracle.so")
    src = os.path.join(_HERE, "oracle.c")
    if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE, "liboracle.so"])
    return so


def lib():
    global _LIB
    if _LIB is None:
        L = ctypes.CDLL(build())
        P, I, D = ctypes.c_void_p, ctypes.c_int, ctypes.c_double
        L.oracle_create.restype = P
        L.oracle_create.argtypes = [P, P, I, P, P, P, P, P, P, P]
        L.oracle_check.argtypes = [P]
        L.oracle_free.argtypes = [P]
        L.oracle_reset.argtypes = [P]
        L.oracle_set_threads.argtypes = [P, I]
        L.oracle_cache_len.argtypes = [P]
        L.oracle_set_cache_len.argtypes = [P, I]
        L.oracle_forward.argtypes = [P, P, I, I, I, P, P]
        L.oracle_generate.argtypes = [P, P, I, I, ctypes.c_int32, P, P, P]
        L.oracle_generate_spec.argtypes = [P, P, I, I, ctypes.c_int32, I, I, P, P, P, P]
        L.oracle_lookup_draft.argtypes = [P, I, I, I, P]
        L.oracle_argmax.argtypes = [P, I]
        L.oracle_argmax_gpt2.argtypes = [P, I, P, I]
        L.oracle_gemv_q4.argtypes = [I, I, P, P, I, P, P, I]
        L.oracle_gemv_q4_f32acc.argtypes = [I, I, P, P, I, P, P]
        _LIB = L
    return _LIB


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def read_pgw(buf: bytes):
    """engine/weights.js:5-40: header fields and the JSON tensor table."""
    if buf[0:4] != b"PGW1":
        raise ValueError("bad magic")
    u32 = lambda o: struct.unpack_from("<I", buf, o)[0]
    f64 = lambda o: struct.unpack_from("<d", buf, o)[0]
    cfg = dict(arch=1 if buf[5] == 1 else 0, vocab=u32(8), n_layers=u32(12), d_model=u32(16), n_heads=u32(20),
               n_kv_heads=u32(24), d_ff=u32(28), max_seq=u32(32), rope_theta=f64(56) or 10000.0,
               rope_pct=f64(64) or 1.0)
    toff, tlen, poff = u32(40), u32(44), u32(48)
    table = json.loads(buf[toff:toff + tlen].decode("utf-8"))
    if cfg["arch"] == 1 and not any(e["name"] == "blocks.0.ln1" for e in table) and \
            any(e["name"] == "blocks.0.norm1" for e in table):
        cfg["arch"] = 0
    return cfg, table, poff


def gemv_q4(packed: np.ndarray, scales: np.ndarray, x: np.ndarray, group: int = 32, threads: int = 1) -> np.ndarray:
    """engine/infer.js:88-116 on one activation row."""
    m = packed.shape[0]
    n = packed.shape[1] * 2
    p = np.ascontiguousarray(packed, np.uint8)
    s = np.ascontiguousarray(scales, np.float32)
    xv = np.ascontiguousarray(x, np.float32)
    y = np.empty(m, np.float32)
    lib().oracle_gemv_q4(m, n, _ptr(p), _ptr(s), group, _ptr(xv), _ptr(y), threads)
    return y


def gemv_q4_f32acc(packed, scales, x, group: int = 32) -> np.ndarray:
    """engine/kernels.rs:60-97 (f32 accumulation)."""
    m = packed.shape[0]
    n = packed.shape[1] * 2
    p = np.ascontiguousarray(packed, np.uint8)
    s = np.ascontiguousarray(scales, np.float32)
    xv = np.ascontiguousarray(x, np.float32)
    y = np.empty(m, np.float32)
    lib().oracle_gemv_q4_f32acc(m, n, _ptr(p), _ptr(s), group, _ptr(xv), _ptr(y))
    return y


def f16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    """f16ToF32 (engine/weights.js:159): IEEE half to float, exact."""
    return np.ascontiguousarray(u16, np.uint16).view(np.float16).astype(np.float32)


def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    """The bf16 conversion of gemvBf16 (engine/infer.js:66-77): the 16 bits become the top of an f32."""
    return (np.ascontiguousarray(u16, np.uint16).astype(np.uint32) << 16).view(np.float32)


def gemv_dense(dtype: str, w: np.ndarray, scales, x: np.ndarray) -> np.ndarray:
    """gemvF32 / gemvF16 / gemvBf16 / gemvQ8 (engine/infer.js:10-86): y[r] = sum_k W[r][k] x[k] in f64
    (the JS `let s` accumulator), stored as f32; q8 multiplies the row sum by the row scale.  w holds
    f32 values, uint16 words (f16 / bf16) or int8 values; x is one activation row."""
    if dtype == "f32":
        wf = np.asarray(w, np.float32).astype(np.float64)
    elif dtype == "f16":
        wf = f16_bits_to_f32(w).astype(np.float64)
    elif dtype == "bf16":
        wf = bf16_bits_to_f32(w).astype(np.float64)
    elif dtype == "q8":
        wf = np.asarray(w, np.int8).astype(np.float64)
    else:
        raise ValueError(dtype)
    y = wf @ np.asarray(x, np.float32).astype(np.float64)
    if dtype == "q8":
        y = y * np.asarray(scales, np.float32).astype(np.float64)
    return y.astype(np.float32)


def lookup_draft(seq, k: int, n: int):
    """engine/webgpu.js:846-865"""
    s = np.ascontiguousarray(seq, np.int32)
    out = np.zeros(max(k, 1), np.int32)
    d = lib().oracle_lookup_draft(_ptr(s), len(s), k, n, _ptr(out))
    return out[:d].tolist()


def argmax_gpt2(logits, history):
    """engine/infer.js:252-287"""
    lg = np.ascontiguousarray(logits, np.float32)
    h = np.ascontiguousarray(history if len(history) else [0], np.int32)
    return lib().oracle_argmax_gpt2(_ptr(lg), len(lg), _ptr(h), len(history))


class OracleModel:
    """engine/infer.js PetitGPT restated in C: forwardPrompt / forwardDecode / generate."""

    def __init__(self, pgw: bytes, threads: int = 1):
        self._buf = np.frombuffer(pgw, np.uint8)
        cfg, table, poff = read_pgw(pgw)
        self.cfg = cfg
        names, st, rows, cols, grp, data, scale = [], [], [], [], [], [], []
        base = self._buf.ctypes.data
        codes = {"f32": 0, "f16": 1, "bf16": 2, "q8": 3, "q4": 4}  # engine/weights.js:3
        for e in table:
            if e["storage"] not in codes:
                raise ValueError(f"unknown tensor storage {e['storage']}")
            names.append(e["name"].encode())
            st.append(codes[e["storage"]])
            shp = e["shape"]
            rows.append(shp[0] if len(shp) == 2 else 1)
            cols.append(shp[1] if len(shp) == 2 else shp[0])
            grp.append(e.get("group") or 32)
            data.append(base + poff + e["offset"])
            scale.append(base + poff + e["scaleOffset"] if e["storage"] in ("q4", "q8") else 0)
        n = len(names)
        cfg_i = np.array([cfg["arch"], cfg["vocab"], cfg["n_layers"], cfg["d_model"], cfg["n_heads"],
                          cfg["n_kv_heads"], cfg["d_ff"], cfg["max_seq"]], np.int32)
        cfg_d = np.array([cfg["rope_theta"], cfg["rope_pct"]], np.float64)
        self._names = (ctypes.c_char_p * n)(*names)
        arr = lambda v, t: np.ascontiguousarray(v, t)
        self._st, self._rows, self._cols, self._grp = (arr(st, np.int32), arr(rows, np.int32), arr(cols, np.int32),
                                                       arr(grp, np.int32))
        self._data = (ctypes.c_void_p * n)(*data)
        self._scale = (ctypes.c_void_p * n)(*[s or None for s in scale])
        self._h = lib().oracle_create(_ptr(cfg_i), _ptr(cfg_d), n, self._names, _ptr(self._st), _ptr(self._rows),
                                      _ptr(self._cols), _ptr(self._grp), self._data, self._scale)
        rc = lib().oracle_check(self._h)
        if rc:
            lib().oracle_free(self._h)
            self._h = None
            raise ValueError(f"PGW file is missing tensors the forward needs (code {rc})")
        lib().oracle_set_threads(self._h, threads)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().oracle_free(self._h)
            self._h = None

    @property
    def vocab(self):
        return self.cfg["vocab"]

    @property
    def cache_len(self):
        return lib().oracle_cache_len(self._h)

    def set_threads(self, n: int):
        lib().oracle_set_threads(self._h, n)

    def reset(self):
        lib().oracle_reset(self._h)

    def forward(self, ids, past_len: int, logits_each: bool = False, hidden: bool = False):
        ids = np.ascontiguousarray(ids, np.int32)
        t = len(ids)
        V = self.vocab
        logits = np.empty((t if logits_each else 1, V), np.float32)
        hid = np.empty((self.cfg["n_layers"], t, self.cfg["d_model"]), np.float32) if hidden else None
        rc = lib().oracle_forward(self._h, _ptr(ids), t, past_len, int(logits_each), _ptr(logits),
                                  _ptr(hid) if hidden else None)
        if rc:
            raise ValueError(f"oracle_forward failed ({rc})")
        out = logits if logits_each else logits[0]
        return (out, hid) if hidden else out

    def forward_prompt(self, ids):
        """engine/infer.js:553-577"""
        self.reset()
        return self.forward(ids, 0)

    def forward_decode(self, tok: int):
        """engine/infer.js:579-601"""
        return self.forward([tok], self.cache_len)

    def generate(self, ids, max_new: int, eos: int = -1, step_logits: bool = False):
        """engine/infer.js:603-646 (prompt truncation applied here, as infer.js:604-608 does)."""
        ids = np.ascontiguousarray(ids, np.int32)
        max_prompt = max(1, self.cfg["max_seq"] - max_new - 1)
        if len(ids) > max_prompt:
            ids = ids[len(ids) - max_prompt:]
        out = np.zeros(max(max_new, 1), np.int32)
        stop = ctypes.c_int(0)
        lg = np.empty((max(max_new, 1), self.vocab), np.float32) if step_logits else None
        n = lib().oracle_generate(self._h, _ptr(ids), len(ids), max_new, eos, _ptr(out), ctypes.byref(stop),
                                  _ptr(lg) if step_logits else None)
        if n < 0:
            raise ValueError(f"oracle_generate failed ({n})")
        res = {"generatedIds": out[:n].tolist(), "stopReason": STOP_NAMES[stop.value]}
        if step_logits:
            res["stepLogits"] = lg[:n]
        return res

    def generate_spec(self, ids, max_new: int, eos: int = -1, spec_k: int = 2, ngram: int = 3):
        """engine/webgpu.js:1164-1282 (fused path with prompt-lookup speculation)."""
        ids = np.ascontiguousarray(ids, np.int32)
        max_prompt = max(1, self.cfg["max_seq"] - max_new - 1)
        if len(ids) > max_prompt:
            ids = ids[len(ids) - max_prompt:]
        out = np.zeros(max(max_new, 1), np.int32)
        stop = ctypes.c_int(0)
        stats = np.zeros(3, np.int32)
        log = np.zeros(max(max_new, 1) * (spec_k + 2) + 8, np.int32)
        n = lib().oracle_generate_spec(self._h, _ptr(ids), len(ids), max_new, eos, spec_k, ngram, _ptr(out),
                                       ctypes.byref(stop), _ptr(stats), _ptr(log))
        if n < 0:
            raise ValueError(f"oracle_generate_spec failed ({n})")
        drafts, pos = [], 0
        for _ in range(int(stats[2])):
            dl = int(log[pos]); pos += 1
            d = log[pos:pos + dl].tolist(); pos += dl
            acc = int(log[pos]); pos += 1
            drafts.append((d, acc))
        return {"generatedIds": out[:n].tolist(), "stopReason": STOP_NAMES[stop.value], "specHits": int(stats[0]),
                "specTries": int(stats[1]), "forwards": int(stats[2]), "drafts": drafts}
