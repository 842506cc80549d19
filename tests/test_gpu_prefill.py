"""Parity of the tensor-core path (tcgen05 GEMMs, flash prefill attention, batched decode) with the oracle
holding the same bf16-rounded weights.

Tolerances (north star, bf16 mode): logits within 2e-2 relative L2; greedy tokens identical."""
import numpy as np
import pytest

from tests.helpers import cfg_dict, native_model, oracle_model, rel_l2, state_dict

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


def oracle_prompt_logits(c, sd, prompt):
    o = oracle_model(c, sd, bf16_weights=True)
    lg = None
    for p, t in enumerate(prompt):
        lg = o.forward_token(int(t), p)
    return o, lg


@pytest.mark.parametrize("variant,batch,plen,page,max_tokens", [
    (dict(), 3, 70, 16, 0),                                        # d 64, page crossings, one chunk
    (dict(head_dim=128, dim=512, heads=4, kv_heads=1), 2, 130, 64, 96),  # d 128, G 4, chunked prompt
    (dict(qk_norm=2, has_qkv_bias=1), 1, 5, 16, 0),                # per-head QK-norm, biases, tiny prompt
    (dict(shared_weights=1, heads=8, kv_heads=8, dim=512), 4, 33, 32, 64),
])
def test_tc_prefill_matches_oracle(variant, batch, plen, page, max_tokens):
    c = cfg_dict(seq_len=160, **variant)
    sd = state_dict(c, seed=21, std=0.05, norm_noise=0.1)
    prompts = np.random.default_rng(22).integers(0, c["vocab"], (batch, plen)).astype(np.int32)
    m = native_model(c, sd, precision="bf16", max_batch=batch, max_tokens=max_tokens or batch * plen, page_size=page)
    lg, am = m.prefill(prompts)
    for b in range(batch):
        o, want = oracle_prompt_logits(c, sd, prompts[b])
        assert rel_l2(lg[b], want) < BF16_TOL, (b, rel_l2(lg[b], want))
        assert am[b] == int(np.argmax(lg[b]))
        # decoding continues from the prefilled cache
        nxt = int(np.argmax(want))
        lg2, _ = m.decode_step([nxt], [plen], slots=[b])
        assert rel_l2(lg2[0], o.forward_token(nxt, plen)) < BF16_TOL
        o.close()
    m.close()


def test_tc_batched_decode_matches_oracle():
    """Eight sequences per step (above the GEMV batch limit): tcgen05 projections with split-K,
    paged decode attention with bf16 output, lm_head GEMM + row argmax."""
    c = cfg_dict(seq_len=64)
    sd = state_dict(c, seed=23, std=0.05, norm_noise=0.1)
    B = 8
    m = native_model(c, sd, precision="bf16", max_batch=B)
    rng = np.random.default_rng(24)
    seqs = rng.integers(0, c["vocab"], (B, 20))
    oracles = [oracle_model(c, sd, bf16_weights=True) for _ in range(B)]
    slots = [5, 2, 7, 0, 1, 6, 3, 4]
    for step in range(20):
        lg, am = m.decode_step(seqs[:, step].tolist(), [step] * B, slots=slots)
        for b in range(B):
            want = oracles[b].forward_token(int(seqs[b, step]), step)
            assert rel_l2(lg[b], want) < BF16_TOL, (step, b)
            assert am[b] == int(np.argmax(lg[b]))
    for o in oracles:
        o.close()


def test_tc_generate_batch_greedy_matches_oracle():
    """Batched prefill + device-resident greedy loop over the tensor-core decode path: six sequences of the
    parity fixture's prompt (tests/golden/tp_parity.npz: N(0, 0.02) synthetic weights, norms 1, a seed whose
    greedy choices all have margins far above the bf16 error) must generate exactly the oracle's 32 tokens."""
    from common_b200 import native
    from tests.tp_worker import parity_fixture
    g, fx = parity_fixture()
    cfg = native.make_config(g["dim"], g["hidden_dim"], g["layers"], g["heads"], g["kv_heads"], g["head_dim"],
                             g["vocab"], g["seq_len"], False, native.QKNORM_VECTOR, False, native.DTYPE_BF16,
                             native.DTYPE_BF16, 6, 48)
    m = native.NativeModel(cfg, 0)
    m.init_synthetic(int(fx["seed"]), float(fx["std"]))
    m.finalize()
    toks = fx["bf16_tokens"]
    got = m.generate(np.repeat(fx["prompt"][None].astype(np.int32), 6, 0), len(toks))
    m.close()
    for b in range(6):
        np.testing.assert_array_equal(got[b], toks)


def test_tc_prefill_8b_layer_geometry():
    """One layer at the Qwen3-8B geometry through the tensor-core prefill: 2 x 200 tokens."""
    c = cfg_dict(dim=4096, hidden_dim=12288, layers=1, heads=32, kv_heads=8, head_dim=128, vocab=8192, seq_len=256)
    sd = state_dict(c, seed=27, std=0.02)
    prompts = np.random.default_rng(28).integers(0, c["vocab"], (2, 200)).astype(np.int32)
    m = native_model(c, sd, precision="bf16", max_batch=2, max_tokens=400)
    lg, _ = m.prefill(prompts)
    for b in range(2):
        o, want = oracle_prompt_logits(c, sd, prompts[b])
        assert rel_l2(lg[b], want) < BF16_TOL
        o.close()


@pytest.mark.parametrize("variant", [dict(), dict(head_dim=128, dim=512, heads=8, kv_heads=1)])
def test_tc_decode_long_context_splits(variant):
    """Five sequences prefilled to 300 positions, then batched decode: the flash-decoding attention splits
    the context across CTAs (up to seq_len/64 splits) and merges them."""
    c = cfg_dict(seq_len=400, **variant)
    sd = state_dict(c, seed=29, std=0.05, norm_noise=0.1)
    B, P = 5, 300
    prompts = np.random.default_rng(30).integers(0, c["vocab"], (B, P)).astype(np.int32)
    m = native_model(c, sd, precision="bf16", max_batch=B, max_tokens=B * P, page_size=32)
    m.prefill(prompts, want_logits=False)
    oracles = []
    for b in range(B):
        o = oracle_model(c, sd, bf16_weights=True)
        for p in range(P):
            o.forward_token(int(prompts[b, p]), p)
        oracles.append(o)
    nxt = np.random.default_rng(31).integers(0, c["vocab"], (3, B))
    for step in range(3):
        lg, _ = m.decode_step(nxt[step].tolist(), [P + step] * B)
        for b in range(B):
            want = oracles[b].forward_token(int(nxt[step, b]), P + step)
            assert rel_l2(lg[b], want) < BF16_TOL, (step, b, rel_l2(lg[b], want))
    for o in oracles:
        o.close()
