"""Tensor parallelism over 2 GPUs (one process per GPU, the library's own NCCL communicator): the
sharded model gives the oracle's logits -- fp32 GEMV decode with the all-reduces after O and down,
the whole-vector QK-norm's all-reduced sums of squares and the distributed argmax; bf16 tensor-core
prefill and batched decode.  Skipped on a box with fewer than 2 GPUs."""
import numpy as np
import pytest

from tests.helpers import cfg_dict, oracle_model, rel_l2, state_dict

pytestmark = pytest.mark.gpu


def _gpus():
    import torch
    return torch.cuda.device_count()


@pytest.mark.skipif("_gpus() < 2")
def test_tp2_matches_oracle():
    import torch.multiprocessing as mp
    from common_b200 import native
    from tests.tp_worker import run_rank
    c = cfg_dict(seq_len=64)
    nids = [native.unique_id() for _ in range(3)]  # one communicator per model
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=run_rank, args=(r, 2, nids, c, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, out, err = q.get(timeout=600)
        assert err is None, err
        res[r] = out
    for p in procs:
        p.join(timeout=120)
    out = res[0]
    sd = state_dict(c, seed=50, std=0.05, norm_noise=0.1)
    toks = np.random.default_rng(51).integers(0, c["vocab"], 24)
    o = oracle_model(c, sd)
    for p, t in enumerate(toks):
        assert rel_l2(out["fp32"][p], o.forward_token(int(t), p)) < 1e-3, p
    o.close()
    prompts = np.random.default_rng(52).integers(0, c["vocab"], (2, 30)).astype(np.int32)
    for b in range(2):
        ob = oracle_model(c, sd, bf16_weights=True)
        want = None
        for p, t in enumerate(prompts[b]):
            want = ob.forward_token(int(t), p)
        assert rel_l2(out["prefill"][b], want) < 2e-2
        ob.close()
    seqs = np.random.default_rng(53).integers(0, c["vocab"], (6, 5))
    for b in range(6):
        ob = oracle_model(c, sd, bf16_weights=True)
        want = None
        for p in range(5):
            want = ob.forward_token(int(seqs[b, p]), p)
        assert rel_l2(out["batch6"][b], want) < 2e-2
        ob.close()
    # greedy tokens of the tensor-parallel step kernel: exactly the oracle's (fixture tp_parity.npz, whose
    # seed leaves every greedy choice a margin far above the bf16 error)
    assert out["step_launches"] == 1
    got = out["greedy"]
    np.testing.assert_array_equal(res[1]["greedy"], got)
    from tests.tp_worker import parity_fixture
    _, fx = parity_fixture()
    np.testing.assert_array_equal(got, fx["bf16_tokens"][:len(got)])
    assert out["graph"] == [int(t) for t in got[9:]]
    # both ranks return the full (gathered) logits
    np.testing.assert_allclose(res[1]["fp32"][5], out["fp32"][5], rtol=1e-5, atol=1e-6)
