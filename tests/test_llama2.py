"""Llama2 checkpoint reading (llama2.c layout, TransformerConfig.java:69-80, Llama2Weights.java:91-115): CPU round
trip and header semantics; on the GPU (marked gpu), the model read from the file against the oracle configured as
the reference's Llama2 (heads = kv heads, no QK-norm, eps 1e-5, the file's RoPE table)."""
import os

import numpy as np
import pytest

from common_b200 import llama2, native
from common_b200.qwen3 import Qwen3Config
from oracle import oracle as O


def tiny_llama(tmp_path, shared=True):
    cfg = Qwen3Config(256, 512, 2, 4, 4, 500, 48, shared, ropeTheta=1e4, qkNorm=native.QKNORM_NONE)
    rng = np.random.default_rng(70)
    D, F, V, L = 256, 512, 500, 2

    def n(*s):
        return (rng.standard_normal(s) * 0.05).astype(np.float32)
    sd = {"model.embed_tokens.weight": n(V, D), "model.norm.weight": 1 + n(D)}
    if not shared:
        sd["lm_head.weight"] = n(V, D)
    for l in range(L):
        p = f"model.layers.{l}."
        sd[p + "input_layernorm.weight"] = 1 + n(D)
        sd[p + "post_attention_layernorm.weight"] = 1 + n(D)
        for k in ("q_proj", "k_proj", "v_proj", "o_proj"):
            sd[p + f"self_attn.{k}.weight"] = n(D, D)
        sd[p + "mlp.gate_proj.weight"] = n(F, D)
        sd[p + "mlp.up_proj.weight"] = n(F, D)
        sd[p + "mlp.down_proj.weight"] = n(D, F)
    # the RoPE table a llama2.c export writes (theta 1e4, float32)
    hs = D // 4
    inv = (1e4 ** (-np.arange(0, hs, 2, dtype=np.float32) / hs)).astype(np.float32)
    ang = np.outer(np.arange(48, dtype=np.float32), inv)
    sd["rope.freq_cis"] = np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32)
    path = os.path.join(str(tmp_path), "model.bin")
    llama2.write_checkpoint(path, cfg, sd)
    return path, cfg, sd


@pytest.mark.parametrize("shared", [True, False])
def test_checkpoint_round_trip(tmp_path, shared):
    path, cfg, sd = tiny_llama(tmp_path, shared)
    cfg2, sd2 = llama2.read_checkpoint(path)
    assert (cfg2.dim, cfg2.hiddenDim, cfg2.layerCount, cfg2.headCount, cfg2.kvHeadCount, cfg2.vocabSize,
            cfg2.seqLen, cfg2.sharedWeights) == (256, 512, 2, 4, 4, 500, 48, shared)
    assert cfg2.headSize == 64 and cfg2.qkNorm == native.QKNORM_NONE
    for k, v in sd.items():
        np.testing.assert_array_equal(sd2.get(k), v)
    assert set(sd2.keySet()) == set(sd.keys())


def test_header_negative_vocab_means_untied(tmp_path):
    path, _, _ = tiny_llama(tmp_path, shared=False)
    assert np.fromfile(path, "<i4", 7)[5] == -500


@pytest.mark.gpu
def test_llama2_on_the_device_matches_oracle(tmp_path):
    path, cfg, sd = tiny_llama(tmp_path, shared=False)
    m = llama2.Llama2(path, precision="fp32")
    got = m.generate([17, 300, 42], 24)[0]
    oc = dict(dim=256, hidden_dim=512, layers=2, heads=4, kv_heads=4, head_dim=64, vocab=500, seq_len=48,
              shared_weights=0, qk_norm=0, has_qkv_bias=0, rope_theta=1e4, eps=1e-5)
    o = O.OracleModel(oc, "f64")
    o.load_state_dict(sd)
    want, _ = o.generate(np.array([1, 17, 300, 42], np.int32), 24)
    np.testing.assert_array_equal(got, want)
    o.close()
    m.close()
