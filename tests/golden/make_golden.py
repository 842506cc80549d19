"""Regenerate tests/golden/tiny_f64.npz: oracle (fp64) logits of the tiny test model for a fixed
token sequence, plus the independent numpy restatement's logits for the same tokens.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, os.path.dirname(HERE))

from oracle import oracle as O  # noqa: E402
from test_oracle import TINY, numpy_forward_model, tiny_state_dict  # noqa: E402


def main():
    sd = tiny_state_dict(TINY)
    toks = np.array([3, 17, 50, 2, 96, 0, 41, 41, 7, 8, 9, 10], np.int32)
    m = O.OracleModel(TINY, "f64")
    m.load_state_dict(sd)
    logits = np.array([m.forward_token(int(t), p) for p, t in enumerate(toks)], np.float32)
    ref = numpy_forward_model(sd, TINY, toks).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "tiny_f64.npz"), tokens=toks, logits=logits, numpy_logits=ref)
    print("max |oracle - numpy|:", float(np.abs(logits - ref).max()))


if __name__ == "__main__":
    main()
