"""The CPU oracle on PGW files whose matrices use the other storage kinds (f32, f16, bf16, q8;
engine/weights.js:3, engine/infer.js:10-86 and 360-420), pinned against an HF transformers float64 Llama
forward of the same weights as engine/weights.js:74-126 decodes them (Bundle.dequant)."""
import numpy as np
import pytest

from conftest import pkg
from oracle import oracle as O

CFG = dict(arch="llama", vocabSize=96, nLayers=2, dModel=128, nHeads=2, nKvHeads=1, dFf=256, maxSeqLen=64,
           ropeTheta=10000.0, std=0.1)


def _hf_llama(b, c):
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM
    d = c["dModel"]
    kv = c["nKvHeads"] * (d // c["nHeads"])
    hc = LlamaConfig(vocab_size=c["vocabSize"], hidden_size=d, intermediate_size=c["dFf"],
                     num_hidden_layers=c["nLayers"], num_attention_heads=c["nHeads"],
                     num_key_value_heads=c["nKvHeads"], max_position_embeddings=c["maxSeqLen"], rms_norm_eps=1e-6,
                     rope_theta=c["ropeTheta"], tie_word_embeddings=False, attention_bias=False, mlp_bias=False)
    m = LlamaForCausalLM(hc).double().eval()
    dq = lambda n: torch.from_numpy(b.dequant(n).astype(np.float64))
    f = lambda n: torch.from_numpy(b.f32(n).astype(np.float64))
    with torch.no_grad():
        m.lm_head.weight.copy_(dq("lm_head"))
        m.model.embed_tokens.weight.copy_(dq("lm_head"))
        for i, L in enumerate(m.model.layers):
            q = dq(f"blocks.{i}.attn.qkv")
            L.self_attn.q_proj.weight.copy_(q[:d])
            L.self_attn.k_proj.weight.copy_(q[d:d + kv])
            L.self_attn.v_proj.weight.copy_(q[d + kv:])
            L.self_attn.o_proj.weight.copy_(dq(f"blocks.{i}.attn.proj"))
            L.mlp.gate_proj.weight.copy_(dq(f"blocks.{i}.mlp.w1"))
            L.mlp.up_proj.weight.copy_(dq(f"blocks.{i}.mlp.w3"))
            L.mlp.down_proj.weight.copy_(dq(f"blocks.{i}.mlp.w2"))
            L.input_layernorm.weight.copy_(f(f"blocks.{i}.norm1"))
            L.post_attention_layernorm.weight.copy_(f(f"blocks.{i}.norm2"))
        m.model.norm.weight.copy_(f("norm_f"))
    return m


@pytest.mark.parametrize("storage", ["f32", "f16", "bf16", "q8"])
def test_oracle_storage_kinds_match_hf_float64(storage):
    import torch
    P = pkg()
    data = P.synthetic_pgw(CFG, 13, storage=storage)
    b = P.parse_pgw(data)
    assert b.tensors["blocks.0.attn.qkv"]["storage"] == storage
    m = _hf_llama(b, CFG)
    om = O.OracleModel(data)
    prompt = P.seeded_prompt(9, CFG["vocabSize"], 5)
    with torch.no_grad():
        hf = m(torch.from_numpy(prompt.astype(np.int64))[None]).logits[0].numpy()
    lg = om.forward(prompt, 0, logits_each=True)
    np.testing.assert_allclose(np.asarray(lg), hf, atol=2e-5, rtol=0)
    # greedy decode continues on the same path (forwardDecode)
    out = om.generate(prompt, 4, eos=-1)
    assert len(out["generatedIds"]) == 4


def test_pgw_storage_kinds_decode_as_the_reference_reads_them():
    """Bundle.dequant (engine/weights.js:74-126) of each storage kind against the writer's rules."""
    P = pkg()
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((5, 64)) * 0.05).astype(np.float32)
    cfg = dict(CFG, vocabSize=5, dModel=64, nLayers=0)
    for storage in ("f32", "f16", "bf16", "q8"):
        b = P.parse_pgw(P.write_pgw(cfg, [("lm_head", w, storage), ("norm_f", np.ones(64, np.float32), "f32")],
                                    kind=storage))
        got = b.dequant("lm_head")
        if storage == "f32":
            want = w
        elif storage == "f16":
            want = w.astype(np.float16).astype(np.float32)
        elif storage == "bf16":
            u = w.view(np.uint32).astype(np.uint64)
            want = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32) << 16).astype(np.uint32).view(np.float32)
        else:
            q, sc = P.quant_q8(w)
            want = q.astype(np.float32) * sc[:, None]
            assert np.abs(got - w).max() <= np.abs(w).max() / 127.0
        np.testing.assert_array_equal(got, want.astype(np.float32))
        assert b.kind == storage


GPT2_CFG = dict(arch="gpt2", vocabSize=80, nLayers=2, dModel=128, nHeads=2, nKvHeads=2, dFf=512, maxSeqLen=64,
                std=0.1)


@pytest.mark.parametrize("storage", ["f16", "q8"])
def test_oracle_gpt2_storage_kinds_match_hf_float64(storage):
    """The GPT-2 path (LayerNorm, biases, tanh GELU, wpe; engine/infer.js:383-392) on f16 and q8 files:
    the embedding takes the stored lm_head row (q8: times its row scale, then / scale_factors)."""
    import torch
    from transformers import GPT2Config, GPT2LMHeadModel
    P = pkg()
    c = GPT2_CFG
    data = P.synthetic_pgw(c, 17, storage=storage)
    b = P.parse_pgw(data)
    d = c["dModel"]
    sf = b.f32("scale_factors").astype(np.float64)
    hc = GPT2Config(vocab_size=c["vocabSize"], n_embd=d, n_head=c["nHeads"], n_layer=c["nLayers"],
                    n_positions=c["maxSeqLen"], tie_word_embeddings=False)
    m = GPT2LMHeadModel(hc).double().eval()
    F = lambda n: torch.from_numpy(b.f32(n).astype(np.float64))
    dq = lambda n: torch.from_numpy(b.dequant(n).astype(np.float64))
    with torch.no_grad():
        lm = dq("lm_head")
        m.lm_head.weight.copy_(lm)
        m.transformer.wte.weight.copy_(lm / torch.from_numpy(sf)[None, :] if storage == "q8" else lm)
        m.transformer.wpe.weight.copy_(F("wpe").reshape(-1, d))
        lnf = F("ln_f")
        m.transformer.ln_f.weight.copy_(lnf[:d])
        m.transformer.ln_f.bias.copy_(lnf[d:])
        for i, blk in enumerate(m.transformer.h):
            ln1, ln2 = F(f"blocks.{i}.ln1"), F(f"blocks.{i}.ln2")
            blk.ln_1.weight.copy_(ln1[:d])
            blk.ln_1.bias.copy_(ln1[d:])
            blk.ln_2.weight.copy_(ln2[:d])
            blk.ln_2.bias.copy_(ln2[d:])
            blk.attn.c_attn.weight.copy_(dq(f"blocks.{i}.attn.qkv").T)
            blk.attn.c_attn.bias.copy_(F(f"blocks.{i}.attn.qkv_bias"))
            blk.attn.c_proj.weight.copy_(dq(f"blocks.{i}.attn.proj").T)
            blk.attn.c_proj.bias.copy_(F(f"blocks.{i}.attn.proj_bias"))
            blk.mlp.c_fc.weight.copy_(dq(f"blocks.{i}.mlp.fc").T)
            blk.mlp.c_fc.bias.copy_(F(f"blocks.{i}.mlp.fc_bias"))
            blk.mlp.c_proj.weight.copy_(dq(f"blocks.{i}.mlp.proj").T)
            blk.mlp.c_proj.bias.copy_(F(f"blocks.{i}.mlp.proj_bias"))
        prompt = P.seeded_prompt(9, c["vocabSize"], 23)
        hf = m(torch.from_numpy(prompt.astype(np.int64))[None]).logits[0].numpy()
    om = O.OracleModel(data)
    lg = om.forward(prompt, 0, logits_each=True)
    np.testing.assert_allclose(np.asarray(lg), hf, atol=5e-5, rtol=0)
