"""The fixture bench.py checks every GPU count against (tests/golden/tp_parity.npz) is the oracle's answer:
regenerate it with the oracle and compare."""
import importlib.util
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def test_tp_parity_fixture_is_the_oracles_answer(tmp_path):
    spec = importlib.util.spec_from_file_location("mk", os.path.join(HERE, "golden", "make_tp_parity.py"))
    mk = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mk)
    want = np.load(os.path.join(HERE, "golden", "tp_parity.npz"))
    mk.main(os.path.join(tmp_path, "tp_parity.npz"))
    got = np.load(os.path.join(tmp_path, "tp_parity.npz"))
    for k in ("prompt", "fp32_logits", "bf16_tokens", "bf16_logits"):
        np.testing.assert_array_equal(got[k], want[k], err_msg=k)
    # greedy choices are the first index of the max of the previous logits
    t, lg = want["bf16_tokens"], want["bf16_logits"].astype(np.float32)
    for p in range(8, len(t)):
        assert t[p] == int(np.argmax(lg[p - 1]))
