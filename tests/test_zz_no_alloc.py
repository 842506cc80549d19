"""qw_op_lm_head_argmax_static: the allocation-free variant of the fused rmsnorm + lm_head +
argmax entry point, for callers that cannot allocate device memory (a JVM passing pointers into
its own pool, a process whose caching allocator must own every byte).  Its scratch is a static
array inside the library, so it must give the same logits and indices as qw_op_lm_head_argmax,
and keep doing so when called twice in a row on the shared array.

Collected last on purpose: a failure here leaves every other test already run."""
import numpy as np
import pytest

from common_b200 import native

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,batch,vocab,dim", [("bf16", 1, 151936, 4096), ("fp32", 4, 5003, 512)])
def test_static_scratch_matches_allocating_entry_point(dtype, batch, vocab, dim):
    import torch
    g = torch.Generator(device="cuda").manual_seed(1)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    wdt = native.DTYPE_BF16 if dtype == "bf16" else native.DTYPE_F32
    W = (torch.randn(vocab, dim, device="cuda", generator=g) * 0.02).to(tdt)
    nw = 1 + 0.1 * torch.randn(dim, device="cuda", generator=g)
    for call in range(2):  # two calls in a row on the shared static scratch, different inputs
        x = torch.randn(batch, dim, device="cuda", generator=g)
        want_l = torch.zeros(batch, vocab, device="cuda")
        want_a = torch.full((batch,), -1, dtype=torch.int32, device="cuda")
        got_l = torch.zeros(batch, vocab, device="cuda")
        got_a = torch.full((batch,), -1, dtype=torch.int32, device="cuda")
        native.op_lm_head_argmax(W.data_ptr(), wdt, vocab, dim, x.data_ptr(), nw.data_ptr(), 1e-6, batch,
                                 want_l.data_ptr(), want_a.data_ptr())
        native.op_lm_head_argmax_static(W.data_ptr(), wdt, vocab, dim, x.data_ptr(), nw.data_ptr(), 1e-6, batch,
                                        got_l.data_ptr(), got_a.data_ptr())
        torch.cuda.synchronize()
        err = ((got_l - want_l).norm() / want_l.norm()).item()
        assert err < 1e-5, (call, err)
        assert np.array_equal(got_a.cpu().numpy(), want_a.cpu().numpy()), call
        lg = got_l.cpu().numpy()
        for b in range(batch):
            assert int(got_a[b]) == int(np.argmax(lg[b]))


def test_static_scratch_entry_rejects_batch_outside_range():
    """batch 5 is outside the op's [1, 4] rows: rejected with QW_ERR_SHAPE before any launch.  (The array's own
    limit, SM count x 8 x batch <= 8192 partials, is out of reach on a 148-SM GPU: 148 x 8 x 4 = 4736.)"""
    with pytest.raises(native.QwenError) as e:
        native.op_lm_head_argmax_static(1, native.DTYPE_F32, 10, 64, 1, 1, 1e-6, 5, 0, 1)
    assert e.value.status == 2
    assert "batch" in str(e.value)
