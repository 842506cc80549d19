"""Token sampling on the device against the restated reference samplers: AutoregressiveModel.sampleToken
(mode 1: temperature, nucleus filter) and the sampler Qwen3 generates with (mode 0: softmax then
sampleToken's second softmax), given the same uniform draws; and sampled generation with the device's
java.util.Random against the oracle drawing from the same seed."""
import numpy as np
import pytest

from common_b200 import native
from oracle import oracle as O
from tests.helpers import cfg_dict, native_model, oracle_model, state_dict

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("vocab,rows", [(151936, 2), (1000, 5)])
@pytest.mark.parametrize("mode,temperature,top_p", [(1, 0.7, 0.9), (1, 1.3, 0.3), (1, 1.0, 1.0), (0, 0.8, 1.0),
                                                    (1, 0.0, 1.0)])
def test_op_sample_matches_reference_sampler(vocab, rows, mode, temperature, top_p):
    import torch
    rng = np.random.default_rng(vocab + rows)
    logits = (rng.standard_normal((rows, vocab)) * 4).astype(np.float32)
    r = rng.random(rows)
    d_lg = torch.tensor(logits, device="cuda")
    d_r = torch.tensor(r, dtype=torch.float64, device="cuda")
    scratch = torch.empty(rows, vocab, dtype=torch.float64, device="cuda")
    out = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
    native.op_sample(d_lg.data_ptr(), rows, vocab, vocab, temperature, top_p, mode, d_r.data_ptr(),
                     scratch.data_ptr(), out.data_ptr())
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b in range(rows):
        if mode == 1:
            want = O.sample_token(logits[b], vocab, temperature, top_p, r[b])
        else:
            want = O.sample_qwen3(logits[b], vocab, temperature, r[b])
        assert got[b] == want, (b, got[b], want)


def test_op_sample_nucleus_ties_in_index_order():
    import torch
    lg = np.full((1, 64), -5.0, np.float32)
    lg[0, [7, 20, 41]] = 3.0  # three equal maxima
    for top_p, r, want in [(0.2, 0.99, 7), (0.5, 0.99, 20), (0.5, 0.1, 7)]:
        d_lg = torch.tensor(lg, device="cuda")
        d_r = torch.tensor([r], dtype=torch.float64, device="cuda")
        scratch = torch.empty(1, 64, dtype=torch.float64, device="cuda")
        out = torch.zeros(1, dtype=torch.int32, device="cuda")
        native.op_sample(d_lg.data_ptr(), 1, 64, 64, 1.0, top_p, 1, d_r.data_ptr(), scratch.data_ptr(), out.data_ptr())
        torch.cuda.synchronize()
        assert int(out.item()) == want == O.sample_token(lg[0], 64, 1.0, top_p, r)


@pytest.mark.parametrize("mode,top_p", [(1, 0.9), (0, 1.0)])
def test_sampled_generation_matches_oracle(mode, top_p):
    """fp32 model: generate with temperature 0.9 draws the oracle's tokens from java.util.Random(seed)."""
    c = cfg_dict(seq_len=48, vocab=300)
    sd = state_dict(c, seed=60, std=0.3, norm_noise=0.1)
    prompt = np.array([5, 17, 2, 200], np.int32)
    m = native_model(c, sd)
    m.set_sampling(0.9, top_p, seed=1234, mode=mode)
    got = m.generate(prompt, 4 + 20)[0]
    o = oracle_model(c, sd)
    jr = O.JavaRandom(1234)
    toks = list(prompt)
    lg = None
    for p in range(4 + 20 - 1):
        lg = o.forward_token(int(toks[p]), p)
        if p >= 3:
            r = jr.next_double()
            nxt = O.sample_token(lg, c["vocab"], 0.9, top_p, r) if mode == 1 else O.sample_qwen3(lg, c["vocab"], 0.9, r)
            toks.append(nxt)
    np.testing.assert_array_equal(got, np.array(toks, np.int32))
    o.close()
    m.close()


def test_decode_sample_host_steps_and_greedy():
    c = cfg_dict(seq_len=32, vocab=300)
    sd = state_dict(c, seed=61, std=0.3)
    m = native_model(c, sd)
    # temperature 0: the same token as the argmax of qw_decode_step
    g = native_model(c, sd)
    for p, t in enumerate([3, 9, 27]):
        _, am = g.decode_step([t], [p])
        assert m.decode_sample([t], [p])[0] == am[0]
    m.reset()
    m.set_sampling(1.1, 0.8, seed=99, mode=1)
    o = oracle_model(c, sd)
    jr = O.JavaRandom(99)
    tok = 3
    for p in range(10):
        got = int(m.decode_sample([tok], [p])[0])
        want = O.sample_token(o.forward_token(tok, p), c["vocab"], 1.1, 0.8, jr.next_double())
        assert got == want, p
        tok = got
    o.close()
    m.close()
    g.close()


def test_qwen3_api_temperature():
    """Qwen3.setTemperature / AutoregressiveModel.next with sampling: the Qwen3 sampler (mode 0) drawing from
    java.util.Random(seed), against the oracle."""
    from common_b200 import Qwen3, Qwen3Config, StateDictionary
    c = cfg_dict(seq_len=32, vocab=300)
    sd = state_dict(c, seed=62, std=0.3)
    cfg = Qwen3Config(c["dim"], c["hidden_dim"], c["layers"], c["heads"], c["kv_heads"], c["vocab"], 32, False,
                      headSize=c["head_dim"])
    q = Qwen3(cfg, StateDictionary(sd), precision="fp32")
    q.setTemperature(0.7, seed=5)
    ar = q.getAutoregressiveModel()
    ar.reset()
    ar.setPrompt([3, 1, 4], 3)
    got = [ar.next() for _ in range(10)]
    o = oracle_model(c, sd)
    jr = O.JavaRandom(5)
    want = [3, 1, 4]
    for p in range(9):
        lg = o.forward_token(want[p], p)
        if p >= 2:
            want.append(O.sample_qwen3(lg, c["vocab"], 0.7, jr.next_double()))
    assert got == want[:10]
    o.close()


def test_op_sample_nucleus_cutoff_at_mass_boundary_is_deterministic():
    """top_p equal to the mass of the 50 largest probabilities (summed in sorted order, as sampleToken does): the
    cutoff sits exactly on a boundary, where a rounding-order-dependent sum could keep one element more or less.
    The device's mass sums are integer (fixed point), so 20 repeated draws give one answer; it is the reference's
    answer just below or just above the boundary, and equals the reference's at 1e-9 relative on either side."""
    import torch
    rng = np.random.default_rng(77)
    V = 151936
    logits = (rng.standard_normal((1, V)) * 3).astype(np.float32)
    p = np.exp(logits[0].astype(np.float64) - logits[0].max())
    p /= p.sum()
    top_p = float(np.sort(p)[::-1][:50].sum())
    r = 0.9999  # the last kept element decides the draw
    d_lg = torch.tensor(logits, device="cuda")
    d_r = torch.tensor([r], dtype=torch.float64, device="cuda")
    scratch = torch.empty(1, V, dtype=torch.float64, device="cuda")

    def draw(tp):
        out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        native.op_sample(d_lg.data_ptr(), 1, V, V, 1.0, tp, 1, d_r.data_ptr(), scratch.data_ptr(), out.data_ptr())
        torch.cuda.synchronize()
        return int(out.item())

    got = {draw(top_p) for _ in range(20)}
    assert len(got) == 1, got
    lo, hi = top_p * (1 - 1e-9), top_p * (1 + 1e-9)
    assert got.pop() in (O.sample_token(logits[0], V, 1.0, lo, r), O.sample_token(logits[0], V, 1.0, hi, r))
    for tp in (lo, hi):
        assert draw(tp) == O.sample_token(logits[0], V, 1.0, tp, r), tp
