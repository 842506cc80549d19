"""The benchmark configurations run as configured, against the oracle.

C1 is the reference's own CPU-runnable case: Qwen3-0.6B geometry (hidden 1024, 28 layers, 16 Q / 8 KV heads,
head_dim 128, intermediate 3072, vocab 151936, tied embeddings, QK-norm, RoPE theta 1e6), fp32 weights
N(0, 0.02) from numpy default_rng(0) with every norm weight 1, a 32-token uniform-random prompt fed one token
per step, then 64 greedy steps, each token the first index of the max of the previous step's logits
(AutoregressiveModel.java:295-308, AggregationFeatures.java:111-121).  fp32 mode: logits within 1e-3 relative
L2 of the fp64 oracle at every one of the 96 positions, and the 64 generated tokens identical."""
import numpy as np
import pytest

from tests.helpers import cfg_dict, native_model, oracle_model, rel_l2, state_dict

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-3

C1 = dict(dim=1024, hidden_dim=3072, layers=28, heads=16, kv_heads=8, head_dim=128, vocab=151936,
          shared_weights=1, qk_norm=1, has_qkv_bias=0, rope_theta=1e6, eps=1e-6)


def test_c1_qwen3_0p6b_fp32_prompt32_greedy64():
    c = cfg_dict(seq_len=128, **C1)
    sd = state_dict(c, seed=0, std=0.02)  # default_rng(0), N(0, 0.02), norms = 1
    prompt = np.random.default_rng(1).integers(0, c["vocab"], 32)
    m = native_model(c, sd, precision="fp32")
    o = oracle_model(c, sd, precision="f64")
    del sd
    tok = int(prompt[0])
    got, want_toks, errs = [], [], []
    want_next = None
    for p in range(32 + 64):
        if p < 32:
            tok = int(prompt[p])
        else:
            # both sides continue from the oracle's own greedy choice, and the device's choice must equal it
            got.append(dev_next)
            want_toks.append(want_next)
            tok = want_next
        lg, am = m.decode_step([tok], [p])
        want = o.forward_token(tok, p)
        errs.append(rel_l2(lg[0], want))
        assert am[0] == int(np.argmax(lg[0]))
        dev_next, want_next = int(am[0]), int(np.argmax(want))
    m.close()
    o.close()
    errs = np.array(errs)
    assert errs.max() < FP32_TOL, (errs.argmax(), errs.max())
    assert got == want_toks, [i for i, (a, b) in enumerate(zip(got, want_toks)) if a != b]


# Qwen2.5 layouts (Q/K/V biases, no QK-norm, Qwen3.java:370-373): the 0.5B shape (hidden 896, 14 Q / 2 KV heads of
# 64: seven query heads per KV head) and the 7B attention shape (hidden 3584, 28 Q / 4 KV heads of 128, G = 7)
QWEN25_05B = dict(dim=896, hidden_dim=4864, heads=14, kv_heads=2, head_dim=64, shared_weights=1, qk_norm=0,
                  has_qkv_bias=1)
QWEN25_7B_CUT = dict(dim=3584, hidden_dim=3584, heads=28, kv_heads=4, head_dim=128, shared_weights=0, qk_norm=0,
                     has_qkv_bias=1)


@pytest.mark.parametrize("shape", [QWEN25_05B, QWEN25_7B_CUT], ids=["qwen2.5-0.5b", "qwen2.5-7b-cut"])
def test_qwen25_shapes_match_oracle(shape):
    c = cfg_dict(layers=2, vocab=4096, seq_len=96, **shape)
    sd = state_dict(c, seed=70, std=0.02)
    toks = np.random.default_rng(71).integers(0, c["vocab"], 40)
    # fp32, batch-1 GEMV path
    m = native_model(c, sd, precision="fp32")
    o = oracle_model(c, sd)
    for p, t in enumerate(toks[:24]):
        lg, _ = m.decode_step([int(t)], [p])
        assert rel_l2(lg[0], o.forward_token(int(t), p)) < FP32_TOL, p
    m.close()
    o.close()
    # bf16: batch-1 decode (the persistent step kernel where the geometry fits it), then tensor-core prefill and
    # batched decode
    ob = oracle_model(c, sd, bf16_weights=True)
    m = native_model(c, sd, precision="bf16", max_batch=6, max_tokens=6 * 32)
    want = []
    for p, t in enumerate(toks[:33]):
        lg, _ = m.decode_step([int(t)], [p])
        want.append(ob.forward_token(int(t), p))
        assert rel_l2(lg[0], want[-1]) < 2e-2, p
    prompts = np.repeat(toks[None, :32].astype(np.int32), 6, 0)
    lg, _ = m.prefill(prompts, slots=np.arange(6, dtype=np.int32))
    for b in range(6):
        assert rel_l2(lg[b], want[31]) < 2e-2, b
    lg2, _ = m.decode_step([int(toks[32])] * 6, [32] * 6)
    for b in range(6):
        assert rel_l2(lg2[b], want[32]) < 2e-2, b
    m.close()
    ob.close()
