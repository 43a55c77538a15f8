#!/usr/bin/env python3
"""Regenerate the golden fixtures in this directory from the reference's own Python code.

Run in a container where the reference project is mounted, with MLLM_REFERENCE_DIR set to its root
(the script stops with an error when it is unset).  It needs torch, transformers and
tokenizers; the tests that read the fixtures need none of them and never read the reference project.

Fixtures:
  q4_pack.npz          float32 matrices (seeded, plus edge cases) and what the reference's
                       quant_q4 (tools/convert_hf_to_pgw.py:18-34) packs them into.
  ref_llama.pgw        a tiny Llama converted by the reference's convert() (tools/convert_hf_to_pgw.py:79-188);
                       its f32 weights come from pgw.llama_tensor_list(REF_LLAMA, seed=11, std=0.1), so
                       the product's writer can be compared byte for byte.
  ref_llama_hf.npz     HF transformers float64 logits of that model (weights dequantised from the
                       file) for a seeded prompt: last-position logits, plus a 6-step greedy rollout.
  ref_gpt2.pgw         a tiny GPT-2 converted by the reference's GPT-2 converter
                       (tools/convert_gpt2_to_pgw.py:83-209), SmoothQuant calibration included.
  ref_gpt2_hf.npz      HF GPT-2 float64 logits of the model the file describes (wte = lm_head rows
                       divided by scale_factors, engine/infer.js:416-419).
"""
from __future__ import annotations

import importlib
import importlib.util
import json
import os
import sys
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("MLLM_REFERENCE_DIR", "")
sys.path.insert(0, ROOT)
pgw = importlib.import_module("microllm-lab_b200.pgw")

# head_dim 64 (the CUDA path's only head size), GQA 2:1
REF_LLAMA = dict(arch="llama", vocabSize=96, nLayers=2, dModel=128, nHeads=2, nKvHeads=1, dFf=128, maxSeqLen=256,
                 ropeTheta=10000.0)
REF_GPT2 = dict(vocab=259, n_embd=128, n_head=2, n_layer=1, n_positions=128)


def load_ref(rel):
    if not REF or not os.path.isdir(REF):
        raise SystemExit("set MLLM_REFERENCE_DIR to the reference project's root directory")
    spec = importlib.util.spec_from_file_location("ref_" + os.path.basename(rel)[:-3], os.path.join(REF, rel))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def wordlevel_tokenizer(vocab: int, path: str):
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    vocab_map = {f"t{i}": i for i in range(vocab)}
    tk = Tokenizer(models.WordLevel(vocab_map, unk_token="t0"))
    tk.pre_tokenizer = pre_tokenizers.Whitespace()
    fast = PreTrainedTokenizerFast(tokenizer_object=tk, unk_token="t0", bos_token="t1", eos_token="t2")
    fast.save_pretrained(path)


def bytelevel_tokenizer(path: str):
    """259-entry byte-level BPE without merges, enough to encode the GPT-2 converter's calibration texts."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    alphabet = pre_tokenizers.ByteLevel.alphabet()
    vocab_map = {ch: i for i, ch in enumerate(sorted(alphabet))}
    for extra in ("<|endoftext|>", "<pad>", "<unk>"):
        vocab_map[extra] = len(vocab_map)
    tk = Tokenizer(models.BPE(vocab_map, [], unk_token="<unk>"))
    tk.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tk.decoder = decoders.ByteLevel()
    fast = PreTrainedTokenizerFast(tokenizer_object=tk, bos_token="<|endoftext|>", eos_token="<|endoftext|>",
                                   unk_token="<unk>")
    fast.save_pretrained(path)
    return len(vocab_map)


def make_q4_pack(ref_cv):
    rng = np.random.default_rng(5)
    cases = {
        "m0": rng.standard_normal((8, 64), dtype=np.float32) * np.float32(0.02),
        "m1": rng.standard_normal((5, 96), dtype=np.float32),
        "m2": (rng.standard_normal((3, 128), dtype=np.float32) * np.float32(3.0)),
    }
    edge = np.zeros((4, 64), np.float32)
    edge[1, :32] = np.linspace(-1.0, 1.0, 32, dtype=np.float32)             # exact amax on both signs
    edge[2, :] = np.tile(np.array([0.5, -0.5, 1.5, 2.5, -8.0, 8.0, 0.0, 7.5], np.float32), 8)  # rint ties
    edge[3, 32:] = np.float32(1e-30)                                         # tiny nonzero group
    cases["edge"] = edge
    out = {}
    for k, m in cases.items():
        packed, scales = ref_cv.quant_q4(m)
        out[k + "_w"], out[k + "_packed"], out[k + "_scales"] = m, packed, scales
    np.savez_compressed(os.path.join(HERE, "q4_pack.npz"), **out)


def dq(b, name):
    return torch.from_numpy(b.dequant(name).astype(np.float64))


def make_llama(ref_cv):
    from transformers import LlamaConfig, LlamaForCausalLM
    c = REF_LLAMA
    tl = pgw.llama_tensor_list(c, 11, std=0.1)
    w = {n: a for n, a, _ in tl}
    d, hd = c["dModel"], c["dModel"] // c["nHeads"]
    kv = c["nKvHeads"] * hd
    hc = LlamaConfig(vocab_size=c["vocabSize"], hidden_size=d, intermediate_size=c["dFf"],
                     num_hidden_layers=c["nLayers"], num_attention_heads=c["nHeads"], num_key_value_heads=c["nKvHeads"],
                     max_position_embeddings=c["maxSeqLen"], rms_norm_eps=1e-6, rope_theta=c["ropeTheta"],
                     tie_word_embeddings=False, attention_bias=False, mlp_bias=False)
    m = LlamaForCausalLM(hc).float().eval()
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    with torch.no_grad():
        m.lm_head.weight.copy_(T(w["lm_head"]))
        m.model.embed_tokens.weight.copy_(T(w["lm_head"]))
        for i, L in enumerate(m.model.layers):
            q = w[f"blocks.{i}.attn.qkv"]
            L.self_attn.q_proj.weight.copy_(T(q[:d]))
            L.self_attn.k_proj.weight.copy_(T(q[d:d + kv]))
            L.self_attn.v_proj.weight.copy_(T(q[d + kv:]))
            L.self_attn.o_proj.weight.copy_(T(w[f"blocks.{i}.attn.proj"]))
            L.mlp.gate_proj.weight.copy_(T(w[f"blocks.{i}.mlp.w1"]))
            L.mlp.up_proj.weight.copy_(T(w[f"blocks.{i}.mlp.w3"]))
            L.mlp.down_proj.weight.copy_(T(w[f"blocks.{i}.mlp.w2"]))
    with tempfile.TemporaryDirectory() as src, tempfile.TemporaryDirectory() as dst:
        m.save_pretrained(src)
        wordlevel_tokenizer(c["vocabSize"], src)
        ref_cv.convert(src, __import__("pathlib").Path(dst), max_seq=c["maxSeqLen"])
        data = open(os.path.join(dst, "model.q4.bin"), "rb").read()
    open(os.path.join(HERE, "ref_llama.pgw"), "wb").write(data)
    # HF float64 forward on the dequantised file
    b = pgw.parse_pgw(data)
    m = m.double()
    with torch.no_grad():
        m.lm_head.weight.copy_(dq(b, "lm_head"))
        m.model.embed_tokens.weight.copy_(dq(b, "lm_head"))
        for i, L in enumerate(m.model.layers):
            q = dq(b, f"blocks.{i}.attn.qkv")
            L.self_attn.q_proj.weight.copy_(q[:d])
            L.self_attn.k_proj.weight.copy_(q[d:d + kv])
            L.self_attn.v_proj.weight.copy_(q[d + kv:])
            L.self_attn.o_proj.weight.copy_(dq(b, f"blocks.{i}.attn.proj"))
            L.mlp.gate_proj.weight.copy_(dq(b, f"blocks.{i}.mlp.w1"))
            L.mlp.up_proj.weight.copy_(dq(b, f"blocks.{i}.mlp.w3"))
            L.mlp.down_proj.weight.copy_(dq(b, f"blocks.{i}.mlp.w2"))
            L.input_layernorm.weight.copy_(torch.from_numpy(b.f32(f"blocks.{i}.norm1").astype(np.float64)))
            L.post_attention_layernorm.weight.copy_(torch.from_numpy(b.f32(f"blocks.{i}.norm2").astype(np.float64)))
        m.model.norm.weight.copy_(torch.from_numpy(b.f32("norm_f").astype(np.float64)))
        prompt = pgw.seeded_prompt(10, c["vocabSize"], 21)
        ids = torch.from_numpy(prompt.astype(np.int64))[None]
        last = m(ids).logits[0, -1].numpy()
        greedy, step_logits = [], []
        cur = ids
        for _ in range(6):
            lg = m(cur).logits[0, -1]
            nxt = int(torch.argmax(lg))
            greedy.append(nxt)
            step_logits.append(lg.numpy())
            cur = torch.cat([cur, torch.tensor([[nxt]])], dim=1)
    np.savez_compressed(os.path.join(HERE, "ref_llama_hf.npz"), prompt=prompt, last_logits=last,
                        greedy=np.array(greedy, np.int32), step_logits=np.stack(step_logits),
                        cfg=json.dumps(c), seed=11, std=0.1)


def make_gpt2(ref_g2):
    from transformers import GPT2Config, GPT2LMHeadModel
    c = REF_GPT2
    with tempfile.TemporaryDirectory() as src, tempfile.TemporaryDirectory() as dst:
        vocab = bytelevel_tokenizer(src)
        assert vocab == c["vocab"], vocab
        hc = GPT2Config(vocab_size=c["vocab"], n_embd=c["n_embd"], n_head=c["n_head"], n_layer=c["n_layer"],
                        n_positions=c["n_positions"], bos_token_id=256, eos_token_id=256)
        torch.manual_seed(13)
        m = GPT2LMHeadModel(hc).float().eval()
        with torch.no_grad():  # make the LayerNorms and biases non-trivial
            for p_name, p in m.named_parameters():
                if "ln_" in p_name or p_name.endswith(".bias"):
                    p.add_(torch.randn_like(p) * 0.1)
        m.save_pretrained(src)
        ref_g2.convert(src, __import__("pathlib").Path(dst))
        data = open(os.path.join(dst, "model.q4.bin"), "rb").read()
    open(os.path.join(HERE, "ref_gpt2.pgw"), "wb").write(data)
    b = pgw.parse_pgw(data)
    d = c["n_embd"]
    sf = b.f32("scale_factors").astype(np.float64)
    hc2 = GPT2Config(vocab_size=c["vocab"], n_embd=d, n_head=c["n_head"], n_layer=c["n_layer"],
                     n_positions=c["n_positions"], tie_word_embeddings=False)
    m2 = GPT2LMHeadModel(hc2).double().eval()
    F = lambda n: torch.from_numpy(b.f32(n).astype(np.float64))
    with torch.no_grad():
        lm = dq(b, "lm_head")
        m2.lm_head.weight.copy_(lm)
        m2.transformer.wte.weight.copy_(lm / torch.from_numpy(sf)[None, :])
        m2.transformer.wpe.weight.copy_(F("wpe").reshape(-1, d))
        lnf = F("ln_f")
        m2.transformer.ln_f.weight.copy_(lnf[:d]); m2.transformer.ln_f.bias.copy_(lnf[d:])
        for i, blk in enumerate(m2.transformer.h):
            ln1, ln2 = F(f"blocks.{i}.ln1"), F(f"blocks.{i}.ln2")
            blk.ln_1.weight.copy_(ln1[:d]); blk.ln_1.bias.copy_(ln1[d:])
            blk.ln_2.weight.copy_(ln2[:d]); blk.ln_2.bias.copy_(ln2[d:])
            blk.attn.c_attn.weight.copy_(dq(b, f"blocks.{i}.attn.qkv").T)
            blk.attn.c_attn.bias.copy_(F(f"blocks.{i}.attn.qkv_bias"))
            blk.attn.c_proj.weight.copy_(dq(b, f"blocks.{i}.attn.proj").T)
            blk.attn.c_proj.bias.copy_(F(f"blocks.{i}.attn.proj_bias"))
            blk.mlp.c_fc.weight.copy_(dq(b, f"blocks.{i}.mlp.fc").T)
            blk.mlp.c_fc.bias.copy_(F(f"blocks.{i}.mlp.fc_bias"))
            blk.mlp.c_proj.weight.copy_(dq(b, f"blocks.{i}.mlp.proj").T)
            blk.mlp.c_proj.bias.copy_(F(f"blocks.{i}.mlp.proj_bias"))
        prompt = pgw.seeded_prompt(9, c["vocab"], 23)
        logits = m2(torch.from_numpy(prompt.astype(np.int64))[None]).logits[0].numpy()
    np.savez_compressed(os.path.join(HERE, "ref_gpt2_hf.npz"), prompt=prompt, logits=logits, cfg=json.dumps(c))


def main():
    ref_cv = load_ref("tools/convert_hf_to_pgw.py")
    ref_g2 = load_ref("tools/convert_gpt2_to_pgw.py")
    make_q4_pack(ref_cv)
    make_llama(ref_cv)
    make_gpt2(ref_g2)
    for f in sorted(os.listdir(HERE)):
        print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
