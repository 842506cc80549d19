"""Bounded device-side waits: a wait that runs out stops the kernel and is reported as QW_ERR_TIMEOUT,
and the CUDA context stays usable.

The persistent decode step separates its phases with grid barriers whose waits are bounded by
qw_config.wait_limit_us.  The test hook qw_config.test_stall_cta makes one CTA withhold its arrival at
the step's first barrier (a count that nothing completes), so every other CTA's wait runs out; no GPU
fault is involved."""
import numpy as np
import pytest

from common_b200 import native
from tests.helpers import cfg_dict, native_model, oracle_model, rel_l2, state_dict

pytestmark = pytest.mark.gpu


def _cfg(c, **kw):
    return native.make_config(c["dim"], c["hidden_dim"], c["layers"], c["heads"], c["kv_heads"], c["head_dim"],
                              c["vocab"], c["seq_len"], c["shared_weights"], c["qk_norm"], c["has_qkv_bias"],
                              native.DTYPE_BF16, native.DTYPE_BF16, 1, **kw)


def test_step_kernel_barrier_wait_runs_out_and_reports_timeout():
    c = cfg_dict(seq_len=32, dim=512, hidden_dim=1024, heads=8, kv_heads=4, head_dim=64)
    sd = state_dict(c, seed=50, std=0.05)
    m = native.NativeModel(_cfg(c, wait_limit_us=20000, test_stall_cta=6), 0)  # 20 ms bound; CTA 5 withholds
    for k, v in sd.items():
        m.load_tensor(k, v)
    m.finalize()
    m.decode_step([3], [0], want_logits=False)
    assert m.last_launch_count == 1  # the persistent step kernel ran
    with pytest.raises(native.QwenError) as ei:
        m.synchronize()
    assert ei.value.status == 6, ei.value  # QW_ERR_TIMEOUT
    assert "site" in str(ei.value)  # the site of the wait that gave up (2: a grid barrier)
    m.close()
    # the context survived: the same weights without the hook decode correctly
    ok = native_model(c, sd, precision="bf16")
    o = oracle_model(c, sd, bf16_weights=True)
    for p, t in enumerate([3, 9, 27]):
        lg, _ = ok.decode_step([t], [p])
        assert rel_l2(lg[0], o.forward_token(t, p)) < 2e-2
    ok.synchronize()
    ok.close()
    o.close()
