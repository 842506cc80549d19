"""Writes tests/golden/tp_parity.npz: the oracle's answers for the parity check that bench.py runs before
timing, at every GPU count (tensor parallelism 1..8).

Model: 2 layers, hidden 1024, 32 Q / 8 KV heads of 128 (the Qwen3-8B attention shape, so that a tp-8 shard
still holds 4 query heads and the persistent step kernel runs), intermediate 4096, vocab 4096, untied
lm_head, whole-vector QK-norm, weights from the library's counter-based synthetic generator (seed 18,
std 0.02, every norm weight 1: the BASELINE weight distribution), which the oracle reproduces bit for bit.
Workload: an 8-token prompt fed one token per step, then 32 greedy steps (AutoregressiveModel.java:295-308).

  fp32_logits  (8, V)   fp64 oracle logits at the prompt positions (fp32 mode: within 1e-3 relative L2)
  bf16_tokens  (40,)    tokens fed at positions 0..39 by the oracle holding bf16-rounded weights
  bf16_logits  (40, V)  its logits at those positions, as float16
               (bf16 mode: within 2e-2 relative L2, tokens identical)

The seed was chosen so that the smallest top-1 / top-2 gap over the 33 greedy choices is 3.3 % of the
logits' standard deviation (a bf16 path's error is a few tenths of a percent of it).

  python tests/golden/make_tp_parity.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

GEOM = dict(dim=1024, hidden_dim=4096, layers=2, heads=32, kv_heads=8, head_dim=128, vocab=4096, seq_len=64,
            shared_weights=0, qk_norm=1, has_qkv_bias=0, rope_theta=1e6, eps=1e-6)
SEED, STD, PROMPT, GEN = 18, 0.02, 8, 32


def main(out=None):
    from oracle import oracle as O
    prompt = np.random.default_rng(SEED).integers(0, GEOM["vocab"], PROMPT).astype(np.int32)
    o = O.OracleModel(GEOM, "f64")
    o.init_synthetic(SEED, STD)
    fp32 = np.stack([o.forward_token(int(t), p) for p, t in enumerate(prompt)])
    o.close()
    o = O.OracleModel(GEOM, "f64")
    o.init_synthetic(SEED, STD)
    o.round_weights_bf16()
    toks, lgs = [], []
    tok = None
    for p in range(PROMPT + GEN):
        tok = int(prompt[p]) if p < PROMPT else tok
        lg = o.forward_token(tok, p)
        toks.append(tok)
        lgs.append(lg)
        tok = int(np.argmax(lg))
    o.close()
    out = out or os.path.join(os.path.dirname(os.path.abspath(__file__)), "tp_parity.npz")
    np.savez_compressed(out,
                        prompt=prompt, fp32_logits=fp32.astype(np.float32), bf16_tokens=np.array(toks, np.int32),
                        bf16_logits=np.stack(lgs).astype(np.float16), seed=SEED, std=STD)


if __name__ == "__main__":
    main()
