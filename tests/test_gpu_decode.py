"""Parity of the CUDA decode path (GEMV + paged attention + lm_head/argmax) with the oracle.

Tolerances (from the task's north star):
  fp32 mode: logits within 1e-3 relative L2 per position;
  bf16 mode: greedy tokens identical, logits within 2e-2 relative L2 per position
             (against the oracle holding the same bf16-rounded weights).
"""
import numpy as np
import pytest

from common_b200 import native
from tests.helpers import cfg_dict, native_model, oracle_model, rel_l2, state_dict

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-3
BF16_TOL = 2e-2


def run_both(c, sd, tokens, precision="fp32", bf16_oracle=False, page_size=64, oracle_precision="f64"):
    m = native_model(c, sd, precision=precision, page_size=page_size)
    o = oracle_model(c, sd, precision=oracle_precision, bf16_weights=bf16_oracle)
    errs = []
    for p, t in enumerate(tokens):
        lg, am = m.decode_step([t], [p])
        want = o.forward_token(t, p)
        errs.append(rel_l2(lg[0], want))
        assert am[0] == int(np.argmax(lg[0])), "device argmax disagrees with its own logits"
    m.close()
    o.close()
    return np.array(errs)


def test_fp32_decode_matches_oracle_across_pages():
    c = cfg_dict(seq_len=150)
    sd = state_dict(c, seed=0, std=0.05, norm_noise=0.1)
    toks = np.random.default_rng(1).integers(0, c["vocab"], 140)
    errs = run_both(c, sd, toks, page_size=16)  # 140 positions cross 9 pages of 16
    assert errs.max() < FP32_TOL, errs.max()


def test_bf16_decode_matches_oracle():
    c = cfg_dict(seq_len=96)
    sd = state_dict(c, seed=2, std=0.05, norm_noise=0.1)
    toks = np.random.default_rng(3).integers(0, c["vocab"], 90)
    errs = run_both(c, sd, toks, precision="bf16", bf16_oracle=True)
    assert errs.max() < BF16_TOL, errs.max()


@pytest.mark.parametrize("variant", [
    dict(qk_norm=0), dict(qk_norm=2), dict(has_qkv_bias=1), dict(head_dim=128, dim=512, heads=4, kv_heads=1),
    dict(heads=8, kv_heads=1, dim=512), dict(heads=2, kv_heads=2, dim=128), dict(shared_weights=1),
    dict(dim=384, heads=8, kv_heads=4, head_dim=64, hidden_dim=768),  # q_dim 512 != dim 384
])
def test_fp32_variants(variant):
    c = cfg_dict(seq_len=40, **variant)
    sd = state_dict(c, seed=4, std=0.05, norm_noise=0.1)
    toks = np.random.default_rng(5).integers(0, c["vocab"], 33)
    errs = run_both(c, sd, toks)
    assert errs.max() < FP32_TOL, (variant, errs.max())


def test_synthetic_init_matches_oracle_generator():
    c = cfg_dict(seq_len=16)
    m = native_model(c, None, synthetic_seed=7)
    o = oracle_model(c, None, synthetic_seed=7)
    for p, t in enumerate([1, 5, 9, 400, 999]):
        lg, _ = m.decode_step([t], [p])
        assert rel_l2(lg[0], o.forward_token(t, p)) < FP32_TOL


def test_forward_hidden_equals_token_path():
    c = cfg_dict(seq_len=16)
    sd = state_dict(c, seed=8)
    a = native_model(c, sd)
    b = native_model(c, sd)
    emb = sd["model.embed_tokens.weight"]
    for p, t in enumerate([3, 4, 5, 6]):
        la, ia = a.decode_step([t], [p])
        lb, ib = b.forward_hidden(emb[t][None], [p])
        np.testing.assert_array_equal(la, lb)
        assert ia[0] == ib[0]


def test_batched_decode_slots_and_positions():
    """Six sequences at different positions in one call (two GEMV passes of <=4 rows)."""
    c = cfg_dict(seq_len=48)
    sd = state_dict(c, seed=9, std=0.05)
    B = 6
    m = native_model(c, sd, max_batch=8)
    rng = np.random.default_rng(10)
    seqs = [rng.integers(0, c["vocab"], 10 + 3 * b) for b in range(B)]
    slots = [7, 0, 3, 5, 1, 2]
    oracles = [oracle_model(c, sd) for _ in range(B)]
    want_last = [None] * B
    for step in range(max(len(s) for s in seqs)):
        idx = [b for b in range(B) if step < len(seqs[b])]
        toks = [int(seqs[b][step]) for b in idx]
        lg, am = m.decode_step(toks, [step] * len(idx), slots=[slots[b] for b in idx])
        for j, b in enumerate(idx):
            want = oracles[b].forward_token(int(seqs[b][step]), step)
            assert rel_l2(lg[j], want) < FP32_TOL
            want_last[b] = want
    for o in oracles:
        o.close()


def test_generate_matches_oracle_greedy():
    c = cfg_dict(seq_len=64, vocab=500)
    sd = state_dict(c, seed=11, std=0.08, norm_noise=0.1)
    prompt = np.random.default_rng(12).integers(0, c["vocab"], 8)
    m = native_model(c, sd)
    o = oracle_model(c, sd)
    got = m.generate(prompt, 48)[0]
    want, _ = o.generate(prompt, 48)
    np.testing.assert_array_equal(got, want)


def test_bf16_generate_tokens_identical_32():
    c = cfg_dict(seq_len=64, vocab=500)
    sd = state_dict(c, seed=13, std=0.08, norm_noise=0.1)
    prompt = np.random.default_rng(14).integers(0, c["vocab"], 8)
    m = native_model(c, sd, precision="bf16")
    o = oracle_model(c, sd, bf16_weights=True)
    got = m.generate(prompt, 8 + 32)[0]
    want, _ = o.generate(prompt, 8 + 32)
    np.testing.assert_array_equal(got, want)


def test_graph_replay_equals_eager_steps():
    import torch
    c = cfg_dict(seq_len=64)
    sd = state_dict(c, seed=15, std=0.08)
    a = native_model(c, sd)
    b = native_model(c, sd)
    for m in (a, b):
        m.reserve(0, 40)
    # eager host steps
    tok, hist = 17, [17]
    for p in range(30):
        _, am = a.decode_step([tok], [p], want_logits=False)
        tok = int(am[0])
        hist.append(tok)
    # device graph: token/position advance on the device
    dt = torch.tensor([17], dtype=torch.int32, device="cuda")
    dp = torch.tensor([0], dtype=torch.int32, device="cuda")
    ds = torch.tensor([0], dtype=torch.int32, device="cuda")
    dam = torch.zeros(1, dtype=torch.int32, device="cuda")
    b.capture_decode(dt.data_ptr(), ds.data_ptr(), dp.data_ptr(), 1, 0, dam.data_ptr())
    got = [17]
    for p in range(30):
        b.replay_decode(1)
        b.synchronize()
        got.append(int(dt.item()))
    assert int(dp.item()) == 30
    assert got == hist


def test_reset_and_slot_reuse():
    c = cfg_dict(seq_len=32)
    sd = state_dict(c, seed=16)
    m = native_model(c, sd, max_batch=2)
    toks = [5, 6, 7, 8]
    first = [m.decode_step([t], [p])[0] for p, t in enumerate(toks)]
    m.reset(0)
    again = [m.decode_step([t], [p])[0] for p, t in enumerate(toks)]
    other = [m.decode_step([t], [p], slots=[1])[0] for p, t in enumerate(toks)]
    np.testing.assert_array_equal(np.array(first), np.array(again))
    np.testing.assert_array_equal(np.array(first), np.array(other))


def test_errors_are_reported():
    c = cfg_dict(seq_len=16)
    sd = state_dict(c, seed=17)
    m = native_model(c, sd, max_batch=2, num_pages=1, page_size=16)
    with pytest.raises(native.QwenError) as e:
        m.decode_step([c["vocab"]], [0])
    assert e.value.status == 1
    with pytest.raises(native.QwenError) as e:
        m.decode_step([1], [16])
    assert e.value.status == 2
    with pytest.raises(native.QwenError) as e:
        m.decode_step([1, 2], [0, 0], slots=[0, 0])
    assert e.value.status == 1
    m.decode_step([1], [0])
    with pytest.raises(native.QwenError) as e:  # the only page belongs to slot 0
        m.decode_step([1], [0], slots=[1])
    assert e.value.status == 3
    # missing weights
    cfg = native.make_config(c["dim"], c["hidden_dim"], 1, c["heads"], c["kv_heads"], c["head_dim"], c["vocab"], 16)
    n = native.NativeModel(cfg)
    with pytest.raises(native.QwenError) as e:
        n.finalize()
    assert e.value.status == 7
    with pytest.raises(native.QwenError) as e:
        n.decode_step([1], [0])
    assert e.value.status == 7
    with pytest.raises(native.QwenError) as e:
        n.load_tensor("model.layers.9.mlp.up_proj.weight", np.zeros(4, np.float32))
    assert e.value.status == 9
    with pytest.raises(native.QwenError) as e:
        n.load_tensor("model.norm.weight", np.zeros(3, np.float32))
    assert e.value.status == 2


def test_qwen3_api_mirror():
    """The reference-facing API (Qwen3 / CompiledModel / AutoregressiveModel) over the library."""
    from common_b200 import Qwen3, Qwen3Config, StateDictionary
    c = cfg_dict(seq_len=32)
    sd = state_dict(c, seed=18, std=0.08)
    cfg = Qwen3Config(c["dim"], c["hidden_dim"], c["layers"], c["heads"], c["kv_heads"], c["vocab"], 32, False,
                      headSize=c["head_dim"])
    q = Qwen3(cfg, StateDictionary(sd), precision="fp32")
    o = oracle_model(c, sd)
    ar = q.getAutoregressiveModel()
    ar.reset()
    ar.setPrompt([3, 1, 4], 3)
    got = [ar.next() for _ in range(12)]
    want, _ = o.generate([3, 1, 4], 12)
    assert got == list(want)
    # CompiledModel.forward with an embedding row at position getPosition()
    q.getAutoregressiveModel().reset()
    o.reset()
    emb = sd["model.embed_tokens.weight"]
    lg = q.getCompiledModel().forward(emb[9][None])
    assert rel_l2(lg[0], o.forward_token(9, 0)) < FP32_TOL


def test_bf16_8b_layer_geometry():
    """One layer at the Qwen3-8B geometry (K = 4096 and 12288 GEMVs, 32/8 heads, d 128)."""
    c = cfg_dict(dim=4096, hidden_dim=12288, layers=1, heads=32, kv_heads=8, head_dim=128, vocab=8192, seq_len=80)
    sd = state_dict(c, seed=19, std=0.02)
    toks = np.random.default_rng(20).integers(0, c["vocab"], 70)
    errs = run_both(c, sd, toks, precision="bf16", bf16_oracle=True)
    assert errs.max() < BF16_TOL, errs.max()
