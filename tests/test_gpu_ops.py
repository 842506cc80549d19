"""Op-level entry points over caller-owned device buffers, checked against a plain PyTorch fp32
reference of the same op (rmsnorm -> W x -> first index of the max)."""
import numpy as np
import pytest

from common_b200 import native

pytestmark = pytest.mark.gpu


def torch_ref(W, x, nw, eps):
    import torch
    Wf = W.float()
    xn = nw * x / torch.sqrt((x * x).sum(-1, keepdim=True) / x.shape[-1] + eps)
    return xn @ Wf.t()


@pytest.mark.parametrize("dtype,batch,vocab,dim", [("bf16", 1, 151936, 4096), ("fp32", 3, 1000, 256),
                                                   ("bf16", 4, 4097, 1024)])
def test_op_lm_head_argmax_matches_torch(dtype, batch, vocab, dim):
    import torch
    g = torch.Generator(device="cuda").manual_seed(0)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    W = (torch.randn(vocab, dim, device="cuda", generator=g) * 0.02).to(tdt)
    x = torch.randn(batch, dim, device="cuda", generator=g)
    nw = 1 + 0.1 * torch.randn(dim, device="cuda", generator=g)
    logits = torch.zeros(batch, vocab, device="cuda")
    am = torch.zeros(batch, dtype=torch.int32, device="cuda")
    wdt = native.DTYPE_BF16 if dtype == "bf16" else native.DTYPE_F32
    native.op_lm_head_argmax(W.data_ptr(), wdt, vocab, dim, x.data_ptr(), nw.data_ptr(), 1e-6, batch,
                             logits.data_ptr(), am.data_ptr())
    torch.cuda.synchronize()
    want = torch_ref(W, x, nw, 1e-6)
    err = ((logits - want).norm() / want.norm()).item()
    assert err < 1e-5, err
    # the index is the first maximum of the logits the kernel itself produced
    got = am.cpu().numpy()
    lg = logits.cpu().numpy()
    for b in range(batch):
        assert got[b] == int(np.argmax(lg[b]))


def test_op_lm_head_argmax_ties_pick_first_index():
    import torch
    vocab, dim = 5000, 64
    W = torch.zeros(vocab, dim, device="cuda")
    W[[17, 999, 4000], 0] = 1.0  # three identical maxima
    x = torch.ones(1, dim, device="cuda")
    nw = torch.ones(dim, device="cuda")
    am = torch.zeros(1, dtype=torch.int32, device="cuda")
    native.op_lm_head_argmax(W.data_ptr(), native.DTYPE_F32, vocab, dim, x.data_ptr(), nw.data_ptr(), 1e-6, 1, 0,
                             am.data_ptr())
    torch.cuda.synchronize()
    assert int(am.item()) == 17


def test_op_lm_head_argmax_rejects_bad_sizes():
    with pytest.raises(native.QwenError) as e:
        native.op_lm_head_argmax(1, native.DTYPE_F32, 10, 64, 1, 1, 1e-6, 5, 0, 1)
    assert e.value.status == 2
    with pytest.raises(native.QwenError) as e:
        native.op_lm_head_argmax(1, native.DTYPE_F32, 10, 60, 1, 1, 1e-6, 1, 0, 1)
    assert e.value.status == 2
    with pytest.raises(native.QwenError) as e:
        native.op_lm_head_argmax(0, native.DTYPE_F32, 10, 64, 1, 1, 1e-6, 1, 0, 1)
    assert e.value.status == 1
