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
