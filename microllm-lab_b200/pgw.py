"""PGW1 weight container: parser, Q4 group-32 packer, writer and seeded synthetic models.

The layout is MicroLLM lab's own and is kept byte-for-byte:

* ``parse_pgw`` follows engine/weights.js:5-40 (header fields, JSON tensor table, arch fallback).
* ``quant_q4`` is a vectorised form of tools/convert_hf_to_pgw.py:18-34: per (row, group of 32)
  ``sc = amax / 8`` (1.0 for an all-zero group), ``q = clip(rint(w / sc) + 8, 0, 15)`` computed in
  float32, byte ``j`` of a group holding element ``2j`` in the low nibble and ``2j + 1`` in the high.
* ``write_pgw`` follows tools/convert_hf_to_pgw.py:37-72 and 123-144 (scales blob before the packed
  blob, table at offset 256, payload 16-byte aligned) and the GPT-2 header of
  tools/convert_gpt2_to_pgw.py:171-178 (arch byte 1, qGroup field 1).
* ``synthetic_llama`` / ``synthetic_gpt2`` draw N(0, 0.02) weights from ``numpy.random.default_rng(seed)``
  in the converters' tensor order (tools/convert_hf_to_pgw.py:104-122,
  tools/convert_gpt2_to_pgw.py:134-164); norm gains are 1, LayerNorm biases 0, linear biases 0,
  GPT-2 ``scale_factors`` 1.  Real checkpoints are not available, so every workload uses these.
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
from dataclasses import dataclass, field

import numpy as np

GROUP = 32
DTYPE_CODE = {0: "f32", 1: "f16", 2: "bf16", 3: "q8", 4: "q4"}  # engine/weights.js:3


@dataclass
class Bundle:
    """What engine/weights.js:39 returns: ``{kind, cfg, tensors, buffer, payloadOff}``."""

    kind: str
    cfg: dict
    tensors: dict
    buffer: bytes
    payload_off: int

    def f32(self, name: str) -> np.ndarray:
        """engine/weights.js:42-47"""
        t = self.tensors.get(name)
        if t is None:
            raise KeyError(f"missing tensor {name}")
        if t["storage"] != "f32":
            raise ValueError(f"{name} is {t['storage']}, not f32")
        return np.frombuffer(self.buffer, np.float32, t["nbytes"] // 4, self.payload_off + t["offset"])

    def u8(self, name: str) -> np.ndarray:
        """engine/weights.js:59-62"""
        t = self.tensors[name]
        return np.frombuffer(self.buffer, np.uint8, t["nbytes"], self.payload_off + t["offset"])

    def scales(self, name: str) -> np.ndarray:
        """engine/weights.js:64-67"""
        t = self.tensors[name]
        return np.frombuffer(self.buffer, np.float32, t["scaleNbytes"] // 4, self.payload_off + t["scaleOffset"])

    def dequant(self, name: str) -> np.ndarray:
        """engine/weights.js:74-126, as float32 [rows, cols]."""
        t = self.tensors[name]
        rows, cols = (1, t["shape"][0]) if len(t["shape"]) == 1 else t["shape"]
        st = t["storage"]
        if st == "f32":
            return self.f32(name).reshape(rows, cols).copy()
        if st in ("f16", "bf16"):
            u = np.frombuffer(self.buffer, np.uint16, t["nbytes"] // 2, self.payload_off + t["offset"])
            if st == "f16":
                return u.view(np.float16).astype(np.float32).reshape(rows, cols)
            return (u.astype(np.uint32) << 16).view(np.float32).reshape(rows, cols)
        if st == "q8":
            q = np.frombuffer(self.buffer, np.int8, t["nbytes"], self.payload_off + t["offset"]).reshape(rows, cols)
            return (q.astype(np.float32) * self.scales(name).reshape(rows, 1)).astype(np.float32)
        if st != "q4":
            raise ValueError(st)
        return dequant_q4(self.u8(name).reshape(rows, cols // 2), self.scales(name).reshape(rows, -1),
                          t.get("group") or GROUP)


def parse_pgw(buffer) -> Bundle:
    """Parse a PGW1 file (engine/weights.js:5-40)."""
    buf = bytes(buffer)
    if len(buf) < 256:
        raise ValueError("truncated PGW1 header")
    magic = buf[0:4].decode("latin-1")
    if magic != "PGW1":
        raise ValueError(f"bad magic {magic}")
    kind = DTYPE_CODE.get(buf[4], "f32")
    arch = "gpt2" if buf[5] == 1 else "llama"
    u32 = lambda off: struct.unpack_from("<I", buf, off)[0]
    f64 = lambda off: struct.unpack_from("<d", buf, off)[0]
    cfg = {
        "arch": arch,
        "vocabSize": u32(8),
        "nLayers": u32(12),
        "dModel": u32(16),
        "nHeads": u32(20),
        "nKvHeads": u32(24),
        "dFf": u32(28),
        "maxSeqLen": u32(32),
        "qGroup": u32(36) or 32,
        "ropeTheta": f64(56) or 10000.0,
        "ropePct": f64(64) or 1.0,
    }
    table_off, table_len, payload_off = u32(40), u32(44), u32(48)
    if table_off + table_len > len(buf):
        raise ValueError("truncated PGW1 tensor table")
    table = json.loads(buf[table_off:table_off + table_len].decode("utf-8"))
    tensors = {e["name"]: e for e in table}
    if cfg["arch"] == "gpt2" and "blocks.0.ln1" not in tensors and "blocks.0.norm1" in tensors:
        cfg["arch"] = "llama"
    return Bundle(kind, cfg, tensors, buf, payload_off)


def quant_q4(mat: np.ndarray, group: int = GROUP):
    """Vectorised tools/convert_hf_to_pgw.py:18-34; returns (packed uint8 [rows, cols/2], scales f32 [rows, ng])."""
    mat = np.ascontiguousarray(mat, dtype=np.float32)
    rows, cols = mat.shape
    if cols % group:
        raise ValueError(f"cols {cols} not divisible by group {group}")
    ng = cols // group
    chunk = mat.reshape(rows, ng, group)
    amax = np.max(np.abs(chunk), axis=2)
    sc = np.where(amax > 0, amax / np.float32(8.0), np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(chunk / sc[:, :, None]) + np.float32(8.0), 0, 15).astype(np.uint8)
    packed = (q[:, :, 0::2] | (q[:, :, 1::2] << 4)).reshape(rows, cols // 2)
    return np.ascontiguousarray(packed), sc


def dequant_q4(packed: np.ndarray, scales: np.ndarray, group: int = GROUP) -> np.ndarray:
    """(nib - 8) * sc per element, float32 (engine/weights.js:106-124)."""
    rows = packed.shape[0]
    lo = (packed & 15).astype(np.int32) - 8
    hi = (packed >> 4).astype(np.int32) - 8
    q = np.empty((rows, packed.shape[1] * 2), np.float32)
    q[:, 0::2] = lo
    q[:, 1::2] = hi
    ng = q.shape[1] // group
    return (q.reshape(rows, ng, group) * scales.reshape(rows, ng, 1)).reshape(rows, -1).astype(np.float32)


def quant_q8(mat: np.ndarray):
    """Symmetric per-row int8 (the layout engine/weights.js:96-105 reads): scale = amax / 127,
    q = clip(rint(w / scale), -127, 127).  Rows of zeros get scale 1."""
    mat = np.ascontiguousarray(mat, dtype=np.float32)
    amax = np.abs(mat).max(axis=1)
    scales = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(mat / scales[:, None]), -127, 127).astype(np.int8)
    return q, scales


def _entries_and_payload(tensors):
    """tools/convert_hf_to_pgw.py:37-72 — returns (table entries, payload bytes)."""
    entries, blobs = [], bytearray()
    for name, arr, storage in tensors:
        if storage == "q4":
            packed, scales = arr if isinstance(arr, tuple) else quant_q4(np.asarray(arr))
            scale_off = len(blobs)
            blobs += scales.tobytes()
            data_off = len(blobs)
            blobs += packed.tobytes()
            entries.append({
                "name": name,
                "shape": [int(packed.shape[0]), int(packed.shape[1] * 2)],
                "kind": "q4",
                "storage": "q4",
                "group": GROUP,
                "scaleOffset": scale_off,
                "scaleNbytes": scales.nbytes,
                "offset": data_off,
                "nbytes": packed.nbytes,
            })
        elif storage == "f32":
            data = np.ascontiguousarray(arr, dtype=np.float32)
            off = len(blobs)
            blobs += data.tobytes()
            entries.append({
                "name": name,
                "shape": list(data.shape),
                "kind": "q4",
                "storage": "f32",
                "offset": off,
                "nbytes": data.nbytes,
            })
        elif storage in ("f16", "bf16"):  # 16-bit words, read as engine/weights.js:82-95 does
            a = np.ascontiguousarray(arr, dtype=np.float32)
            if storage == "f16":
                words = a.astype(np.float16).view(np.uint16)
            else:  # round to nearest even on the top 16 bits
                u = a.view(np.uint32).astype(np.uint64)
                words = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
            off = len(blobs)
            blobs += words.tobytes()
            entries.append({"name": name, "shape": list(a.shape), "kind": storage, "storage": storage,
                            "offset": off, "nbytes": words.nbytes})
        elif storage == "q8":  # int8 rows and one f32 scale per row (engine/weights.js:96-105)
            if isinstance(arr, tuple):
                q, scales = arr
            else:
                q, scales = quant_q8(np.asarray(arr))
            scale_off = len(blobs)
            blobs += scales.tobytes()
            data_off = len(blobs)
            blobs += q.tobytes()
            entries.append({"name": name, "shape": [int(q.shape[0]), int(q.shape[1])], "kind": "q8",
                            "storage": "q8", "scaleOffset": scale_off, "scaleNbytes": scales.nbytes,
                            "offset": data_off, "nbytes": q.nbytes})
        else:
            raise ValueError(storage)
    return entries, bytes(blobs)


def write_pgw(cfg: dict, tensors, path: str | None = None, kind: str = "q4") -> bytes:
    """Serialise a PGW1 file (tools/convert_hf_to_pgw.py:123-144; GPT-2 header
    tools/convert_gpt2_to_pgw.py:171-178).  ``tensors`` is a list of (name, array, storage) where a
    q4 array may also be a precomputed (packed, scales) tuple and a q8 array a (q, scales) tuple;
    ``kind`` is the header's dtype byte (engine/weights.js:14)."""
    entries, payload = _entries_and_payload(tensors)
    table = json.dumps(entries, separators=(",", ":")).encode("utf-8")
    table_off = 256
    pad = (16 - ((table_off + len(table)) % 16)) % 16
    payload_off = table_off + len(table) + pad
    gpt2 = cfg.get("arch") == "gpt2"
    header = bytearray(256)
    header[0:4] = b"PGW1"
    header[4] = {v: k for k, v in DTYPE_CODE.items()}[kind]
    header[5] = 1 if gpt2 else 0
    struct.pack_into("<8I", header, 8, cfg["vocabSize"], cfg["nLayers"], cfg["dModel"], cfg["nHeads"],
                     cfg["nKvHeads"], cfg["dFf"], cfg["maxSeqLen"], 1 if gpt2 else GROUP)
    struct.pack_into("<III", header, 40, table_off, len(table), payload_off)
    struct.pack_into("<d", header, 56, 10000.0 if gpt2 else float(cfg.get("ropeTheta", 10000.0)))
    struct.pack_into("<d", header, 64, 1.0)
    out = bytes(header) + table + b"\x00" * pad + payload
    if path is not None:
        with open(path, "wb") as f:
            f.write(out)
    return out


# ----------------------------------------------------------------------------------------------
# Seeded synthetic models (real checkpoints are git-LFS stubs in the reference)
# ----------------------------------------------------------------------------------------------

CONFIGS = {
    # models/petitgpt/card.json
    "petitgpt": dict(arch="llama", vocabSize=32000, nLayers=30, dModel=576, nHeads=9, nKvHeads=3, dFf=1536,
                     maxSeqLen=2048, ropeTheta=10000.0),
    # models/smollm2-135m-instruct/card.json
    "smollm2-135m": dict(arch="llama", vocabSize=49152, nLayers=30, dModel=576, nHeads=9, nKvHeads=3, dFf=1536,
                         maxSeqLen=2048, ropeTheta=100000.0),
    # models/smollm2-360m-instruct/card.json
    "smollm2-360m": dict(arch="llama", vocabSize=49152, nLayers=32, dModel=960, nHeads=15, nKvHeads=5, dFf=2560,
                         maxSeqLen=2048, ropeTheta=100000.0),
    # models/gpt2/card.json
    "gpt2": dict(arch="gpt2", vocabSize=50257, nLayers=12, dModel=768, nHeads=12, nKvHeads=12, dFf=3072,
                 maxSeqLen=1024),
    # Small shapes with the real head_dim (64) for fast parity tests.  Their weights use std 0.1: at
    # 0.02 a random tied-embedding model falls into a one-token attractor after the first step, which
    # makes a token-stream comparison weak.  BASELINE workloads keep 0.02.
    "tiny-llama": dict(arch="llama", vocabSize=512, nLayers=2, dModel=192, nHeads=3, nKvHeads=1, dFf=320,
                       maxSeqLen=160, ropeTheta=10000.0, std=0.1),
    # More query heads per kv head (6) than the token-batch engine takes (4): prefill, verify and
    # multi-token forwards run on the persistent decode_kernel for such files.
    "tiny-llama-r6": dict(arch="llama", vocabSize=512, nLayers=2, dModel=384, nHeads=6, nKvHeads=1, dFf=512,
                          maxSeqLen=160, ropeTheta=10000.0, std=0.1),
    "tiny-gpt2": dict(arch="gpt2", vocabSize=640, nLayers=2, dModel=128, nHeads=2, nKvHeads=2, dFf=512,
                      maxSeqLen=128, std=0.1),
}


def _normal(rng, shape, std=0.02):
    return rng.standard_normal(shape, dtype=np.float32) * np.float32(std)


def llama_tensor_list(cfg: dict, seed: int, std: float = 0.02, storage: str = "q4"):
    """Tensors in tools/convert_hf_to_pgw.py:104-122 order, N(0, std) weights stored as ``storage``,
    unit norm gains."""
    rng = np.random.default_rng(seed)
    d, ff, V = cfg["dModel"], cfg["dFf"], cfg["vocabSize"]
    hd = d // cfg["nHeads"]
    kv = cfg["nKvHeads"] * hd
    out = [("lm_head", _normal(rng, (V, d), std), storage)]
    ones = np.ones(d, np.float32)
    for i in range(cfg["nLayers"]):
        out.append((f"blocks.{i}.norm1", ones, "f32"))
        out.append((f"blocks.{i}.attn.qkv", _normal(rng, (d + 2 * kv, d), std), storage))
        out.append((f"blocks.{i}.attn.proj", _normal(rng, (d, d), std), storage))
        out.append((f"blocks.{i}.norm2", ones, "f32"))
        out.append((f"blocks.{i}.mlp.w1", _normal(rng, (ff, d), std), storage))
        out.append((f"blocks.{i}.mlp.w3", _normal(rng, (ff, d), std), storage))
        out.append((f"blocks.{i}.mlp.w2", _normal(rng, (d, ff), std), storage))
    out.append(("norm_f", ones, "f32"))
    return out


def gpt2_tensor_list(cfg: dict, seed: int, std: float = 0.02, storage: str = "q4"):
    """Tensors in tools/convert_gpt2_to_pgw.py:134-164 order (weights stored as ``storage``);
    scale_factors 1, LN [1; 0], biases 0."""
    rng = np.random.default_rng(seed)
    d, ff, V, ms = cfg["dModel"], cfg["dFf"], cfg["vocabSize"], cfg["maxSeqLen"]
    ln = np.concatenate([np.ones(d, np.float32), np.zeros(d, np.float32)])
    out = [("scale_factors", np.ones(d, np.float32), "f32"),
           ("lm_head", _normal(rng, (V, d), std), storage),
           ("wpe", _normal(rng, (ms, d), std), "f32"),
           ("ln_f", ln, "f32")]
    for i in range(cfg["nLayers"]):
        out.append((f"blocks.{i}.ln1", ln, "f32"))
        out.append((f"blocks.{i}.attn.qkv", _normal(rng, (3 * d, d), std), storage))
        out.append((f"blocks.{i}.attn.qkv_bias", np.zeros(3 * d, np.float32), "f32"))
        out.append((f"blocks.{i}.attn.proj", _normal(rng, (d, d), std), storage))
        out.append((f"blocks.{i}.attn.proj_bias", np.zeros(d, np.float32), "f32"))
        out.append((f"blocks.{i}.ln2", ln, "f32"))
        out.append((f"blocks.{i}.mlp.fc", _normal(rng, (ff, d), std), storage))
        out.append((f"blocks.{i}.mlp.fc_bias", np.zeros(ff, np.float32), "f32"))
        out.append((f"blocks.{i}.mlp.proj", _normal(rng, (d, ff), std), storage))
        out.append((f"blocks.{i}.mlp.proj_bias", np.zeros(d, np.float32), "f32"))
    return out


def synthetic_pgw(name_or_cfg, seed: int, cache_dir: str | None = None, storage: str = "q4") -> bytes:
    """Seeded synthetic PGW1 file for a named config (see CONFIGS) or an explicit cfg dict, its matrices
    stored as ``storage`` (q4 by default; f32 / f16 / bf16 / q8 for the other kinds).  When
    ``cache_dir`` is given the file is cached there under a hash of (cfg, seed, storage)."""
    cfg = dict(CONFIGS[name_or_cfg]) if isinstance(name_or_cfg, str) else dict(name_or_cfg)
    key = hashlib.sha1(json.dumps([cfg, seed] if storage == "q4" else [cfg, seed, storage],
                                  sort_keys=True).encode()).hexdigest()[:16]
    path = None
    if cache_dir:
        os.makedirs(cache_dir, exist_ok=True)
        path = os.path.join(cache_dir, f"synth-{key}.pgw")
        if os.path.exists(path):
            with open(path, "rb") as f:
                return f.read()
    std = float(cfg.get("std", 0.02))
    tl = (gpt2_tensor_list(cfg, seed, std, storage) if cfg["arch"] == "gpt2"
          else llama_tensor_list(cfg, seed, std, storage))
    data = write_pgw(cfg, tl, kind=storage)
    if path:
        tmp = path + f".tmp{os.getpid()}"
        with open(tmp, "wb") as f:
            f.write(data)
        os.replace(tmp, path)
    return data


def seeded_prompt(n: int, vocab: int, seed: int) -> np.ndarray:
    """Uniform token ids in [0, vocab) from default_rng(seed) (3, 5)."""
    return np.random.default_rng(seed).integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)


def copy_span_prompt(n: int, vocab: int, seed: int, span: int = 32) -> np.ndarray:
    """BASELINE config 4 prompt: n seeded ids in which every odd ``span``-token block (half of the
    positions) is a copy of an earlier random ``span``-token span, so that n-gram lookups find matches."""
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)
    for b in range(1, n // span, 2):
        pos = b * span
        src = int(rng.integers(0, pos - span + 1))
        ids[pos:pos + span] = ids[src:src + span]
    return ids
