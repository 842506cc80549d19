"""The tcgen05/TMEM GEMM (qw_op_linear) against a plain PyTorch fp32 reference of the same op on the
same bf16 operands: y = x W^T with the STORE(+bias), RESID and SWIGLU epilogues."""
import pytest

from common_b200 import native

pytestmark = pytest.mark.gpu


def operands(n_out, k, t, seed=0):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    W = (torch.randn(n_out, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    X = torch.randn(t, k, device="cuda", generator=g).to(torch.bfloat16)
    return W, X


def rel(a, b):
    return ((a - b).norm() / b.norm()).item()


# token tiles of 64 / 128 / 256, ragged edges in every dimension, k not a multiple of 64
@pytest.mark.parametrize("n_out,k,t", [(256, 256, 64), (384, 512, 100), (6144, 4096, 512), (200, 136, 3),
                                       (1024, 1024, 300), (128, 64, 1), (4096, 12288, 16)])
def test_linear_store_matches_torch(n_out, k, t):
    import torch
    W, X = operands(n_out, k, t)
    bias = torch.randn(n_out, device="cuda")
    out = torch.full((t, n_out), float("nan"), device="cuda")
    native.op_linear(W.data_ptr(), n_out, k, X.data_ptr(), t, native.LINEAR_STORE, bias.data_ptr(), 0,
                     out.data_ptr())
    torch.cuda.synchronize()
    want = X.float() @ W.float().t() + bias
    assert rel(out, want) < 1e-4  # fp32 accumulation order over k up to 12288


def test_linear_resid_in_place():
    import torch
    n_out, k, t = 512, 1024, 77
    W, X = operands(n_out, k, t, seed=1)
    x = torch.randn(t, n_out, device="cuda")
    want = x + X.float() @ W.float().t()
    native.op_linear(W.data_ptr(), n_out, k, X.data_ptr(), t, native.LINEAR_RESID, 0, x.data_ptr(), x.data_ptr())
    torch.cuda.synchronize()
    assert rel(x, want) < 1e-5


@pytest.mark.parametrize("n_out,t", [(512, 40), (2048, 260)])
def test_linear_swiglu_interleaved(n_out, t):
    import torch
    k = 256
    W, X = operands(n_out, k, t, seed=2)
    out = torch.zeros(t, n_out // 2, dtype=torch.bfloat16, device="cuda")
    native.op_linear(W.data_ptr(), n_out, k, X.data_ptr(), t, native.LINEAR_SWIGLU, 0, 0, out.data_ptr())
    torch.cuda.synchronize()
    y = X.float() @ W.float().t()  # (t, n_out), rows interleaved 16 gate / 16 up
    y = y.view(t, n_out // 32, 2, 16)
    gate, up = y[:, :, 0, :].reshape(t, -1), y[:, :, 1, :].reshape(t, -1)
    want = up * torch.nn.functional.silu(gate)
    assert rel(out.float(), want) < 1e-2  # bf16 output rounding


def test_linear_rejects_bad_shapes():
    with pytest.raises(native.QwenError) as e:
        native.op_linear(16, 64, 12, 16, 4, native.LINEAR_STORE, 0, 0, 16)
    assert e.value.status == 2


# prefill shapes (>= 74 tiles of 256 x 256): the CTA-pair (cta_group::2) kernel, with a ragged token edge, k not a
# multiple of 64 and feature counts whose last 256-row tile is partly or (for the odd CTA) wholly past the end
@pytest.mark.parametrize("n_out,k,t", [(6144, 4096, 4096), (4000, 520, 2500), (4224, 200, 4700)])
def test_linear_pair_store_matches_torch(n_out, k, t):
    import torch
    W, X = operands(n_out, k, t, seed=3)
    bias = torch.randn(n_out, device="cuda")
    out = torch.full((t, n_out), float("nan"), device="cuda")
    native.op_linear(W.data_ptr(), n_out, k, X.data_ptr(), t, native.LINEAR_STORE, bias.data_ptr(), 0,
                     out.data_ptr())
    torch.cuda.synchronize()
    want = X.float() @ W.float().t() + bias
    assert rel(out, want) < 1e-4


def test_linear_pair_resid_in_place():
    import torch
    n_out, k, t = 4096, 1024, 4700
    W, X = operands(n_out, k, t, seed=4)
    x = torch.randn(t, n_out, device="cuda")
    want = x + X.float() @ W.float().t()
    native.op_linear(W.data_ptr(), n_out, k, X.data_ptr(), t, native.LINEAR_RESID, 0, x.data_ptr(), x.data_ptr())
    torch.cuda.synchronize()
    assert rel(x, want) < 1e-5


@pytest.mark.parametrize("n_out,t", [(8192, 2600), (4224, 4700)])
def test_linear_pair_swiglu_interleaved(n_out, t):
    import torch
    k = 512
    W, X = operands(n_out, k, t, seed=5)
    out = torch.zeros(t, n_out // 2, dtype=torch.bfloat16, device="cuda")
    native.op_linear(W.data_ptr(), n_out, k, X.data_ptr(), t, native.LINEAR_SWIGLU, 0, 0, out.data_ptr())
    torch.cuda.synchronize()
    y = (X.float() @ W.float().t()).view(t, n_out // 32, 2, 16)
    gate, up = y[:, :, 0, :].reshape(t, -1), y[:, :, 1, :].reshape(t, -1)
    want = up * torch.nn.functional.silu(gate)
    assert rel(out.float(), want) < 1e-2
