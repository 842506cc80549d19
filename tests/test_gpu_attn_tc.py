"""Causal prefill attention on tcgen05 (head_dim 128): every GQA group size, page sizes below, at and above
the 128-key block, prompts chunked at positions that are not multiples of the query tile.  Checked against
the oracle holding the same bf16-rounded weights (bf16 tolerance 2e-2 relative L2 on the logits) and, more
tightly, against the mma.sync flash kernel on the same weights (QW_TC_ATTN=0 at model creation)."""
import os

import numpy as np
import pytest

from tests.helpers import cfg_dict, native_model, oracle_model, rel_l2, state_dict

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


def _model(c, sd, tc, **kw):
    old = os.environ.get("QW_TC_ATTN")
    os.environ["QW_TC_ATTN"] = "1" if tc else "0"
    try:
        return native_model(c, sd, precision="bf16", **kw)
    finally:
        if old is None:
            del os.environ["QW_TC_ATTN"]
        else:
            os.environ["QW_TC_ATTN"] = old


@pytest.mark.parametrize("heads,kv_heads,page,batch,plen,max_tokens", [
    (4, 4, 64, 2, 300, 0),     # G 1: 128 positions per tile
    (4, 2, 16, 3, 150, 0),     # G 2, 16-token pages (8 boxes per key block)
    (8, 2, 256, 2, 260, 0),    # G 4, a key block inside one 256-token page
    (8, 1, 64, 2, 270, 160),   # G 8, chunks of 80 positions: tiles straddle key blocks
])
def test_tc_attention_prefill_matches_oracle_and_mma_kernel(heads, kv_heads, page, batch, plen, max_tokens):
    c = cfg_dict(dim=512, hidden_dim=1024, heads=heads, kv_heads=kv_heads, head_dim=128, seq_len=320)
    sd = state_dict(c, seed=60, std=0.05, norm_noise=0.1)
    prompts = np.random.default_rng(61).integers(0, c["vocab"], (batch, plen)).astype(np.int32)
    mt = max_tokens or batch * plen
    a = _model(c, sd, True, max_batch=batch, max_tokens=mt, page_size=page)
    b = _model(c, sd, False, max_batch=batch, max_tokens=mt, page_size=page)
    la, _ = a.prefill(prompts)
    lb, _ = b.prefill(prompts)
    a.synchronize()
    for i in range(batch):
        # two bf16 kernels with different P roundings and summation orders: close, not equal
        assert rel_l2(la[i], lb[i]) < 1.5e-2, (i, rel_l2(la[i], lb[i]))
    for i in (0, batch - 1):
        o = oracle_model(c, sd, bf16_weights=True)
        want = None
        for p, t in enumerate(prompts[i]):
            want = o.forward_token(int(t), p)
        ea, eb = rel_l2(la[i], want), rel_l2(lb[i], want)
        print(f"tc attention rel-L2 {ea:.3e}, mma.sync {eb:.3e}")
        assert ea < BF16_TOL, (i, ea, eb)
        assert ea < 1.5 * eb + 2e-3, (i, ea, eb)  # no worse than the kernel it replaces
        o.close()
    a.close()
    b.close()
