"""PGW1 container and Q4 pack: the product's writer/parser against the reference's own converter output."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, pkg


def test_quant_q4_matches_reference_converter():
    """pgw.quant_q4 == tools/convert_hf_to_pgw.py:18-34 on seeded and edge-case matrices."""
    P = pkg()
    z = np.load(os.path.join(GOLDEN, "q4_pack.npz"))
    names = sorted({k.rsplit("_", 1)[0] for k in z.files})
    assert names
    for k in names:
        packed, scales = P.quant_q4(z[k + "_w"])
        np.testing.assert_array_equal(packed, z[k + "_packed"], err_msg=k)
        np.testing.assert_array_equal(scales.view(np.uint32), z[k + "_scales"].view(np.uint32), err_msg=k)


def test_writer_is_byte_identical_to_reference_converter():
    """write_pgw(llama_tensor_list(cfg, 11, 0.1)) reproduces the file the reference converter wrote."""
    P = pkg()
    ref = open(os.path.join(GOLDEN, "ref_llama.pgw"), "rb").read()
    meta = np.load(os.path.join(GOLDEN, "ref_llama_hf.npz"))
    cfg = json.loads(str(meta["cfg"]))
    tl = P.pgw.llama_tensor_list(cfg, int(meta["seed"]), std=float(meta["std"]))
    mine = P.write_pgw(cfg, tl)
    assert mine == ref


def test_parse_reference_files():
    P = pkg()
    b = P.parse_pgw(open(os.path.join(GOLDEN, "ref_llama.pgw"), "rb").read())
    assert b.kind == "q4" and b.cfg["arch"] == "llama"
    assert (b.cfg["vocabSize"], b.cfg["nLayers"], b.cfg["dModel"], b.cfg["nHeads"], b.cfg["nKvHeads"]) == (96, 2, 128, 2, 1)
    assert b.payload_off % 16 == 0
    g = P.parse_pgw(open(os.path.join(GOLDEN, "ref_gpt2.pgw"), "rb").read())
    assert g.cfg["arch"] == "gpt2" and g.cfg["qGroup"] == 1 and g.cfg["nKvHeads"] == g.cfg["nHeads"]
    assert "scale_factors" in g.tensors and g.tensors["ln_f"]["shape"] == [2 * g.cfg["dModel"]]


def test_parse_errors():
    P = pkg()
    good = open(os.path.join(GOLDEN, "ref_llama.pgw"), "rb").read()
    with pytest.raises(ValueError, match="bad magic"):
        P.parse_pgw(b"PGW2" + good[4:])
    with pytest.raises(ValueError, match="truncated"):
        P.parse_pgw(good[:100])


def test_synthetic_sizes_match_model_cards():
    """Header + table + payload of the synthetic PetitGPT file equal the real card's q4Bytes (78,046,720)."""
    P = pkg()
    cfg = dict(P.CONFIGS["petitgpt"])
    d, ff, V, L = cfg["dModel"], cfg["dFf"], cfg["vocabSize"], cfg["nLayers"]
    kv = cfg["nKvHeads"] * (d // cfg["nHeads"])
    q4 = lambda r, c: r * c // 2 + r * (c // 32) * 4
    payload = q4(V, d) + L * (2 * d * 4 + q4(d + 2 * kv, d) + q4(d, d) + 2 * q4(ff, d) + q4(d, ff)) + d * 4
    # table: build it with tiny zero arrays of the right shapes is too big; compare payload and the
    # table length the writer would produce for the same entries.
    entries = []
    off = 0
    for name, shp, st in ([("lm_head", (V, d), "q4")] + sum([[
            (f"blocks.{i}.norm1", (d,), "f32"), (f"blocks.{i}.attn.qkv", (d + 2 * kv, d), "q4"),
            (f"blocks.{i}.attn.proj", (d, d), "q4"), (f"blocks.{i}.norm2", (d,), "f32"),
            (f"blocks.{i}.mlp.w1", (ff, d), "q4"), (f"blocks.{i}.mlp.w3", (ff, d), "q4"),
            (f"blocks.{i}.mlp.w2", (d, ff), "q4")] for i in range(L)], []) + [("norm_f", (d,), "f32")]):
        if st == "q4":
            sn = shp[0] * (shp[1] // 32) * 4
            entries.append({"name": name, "shape": list(shp), "kind": "q4", "storage": "q4", "group": 32,
                            "scaleOffset": off, "scaleNbytes": sn, "offset": off + sn, "nbytes": shp[0] * shp[1] // 2})
            off += sn + shp[0] * shp[1] // 2
        else:
            entries.append({"name": name, "shape": list(shp), "kind": "q4", "storage": "f32", "offset": off,
                            "nbytes": shp[0] * 4})
            off += shp[0] * 4
    assert off == payload
    table = json.dumps(entries, separators=(",", ":")).encode()
    total = 256 + len(table) + (16 - (256 + len(table)) % 16) % 16 + payload
    assert total == 78_046_720


def test_copy_span_prompt_has_matches():
    P = pkg()
    ids = P.copy_span_prompt(512, 49152, 3)
    assert len(ids) == 512 and ids.dtype == np.int32
    copied = 0
    for b in range(1, 16, 2):
        blk = ids[b * 32:(b + 1) * 32]
        src = [i for i in range(0, b * 32 - 31) if np.array_equal(ids[i:i + 32], blk)]
        copied += bool(src)
    assert copied == 8
