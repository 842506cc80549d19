"""One tensor-parallel rank of the GPU TP tests (run in a spawned process per GPU).  Every model gets its
own NCCL unique id: an id bootstraps exactly one communicator."""
import numpy as np


def run_rank(rank, world, nids, c, q):
    try:
        from common_b200 import native
        from tests.helpers import native_model_tp, state_dict
        out = {}
        sd = state_dict(c, seed=50, std=0.05, norm_noise=0.1)
        toks = np.random.default_rng(51).integers(0, c["vocab"], 24)
        # fp32, batch 1, GEMV path with the all-reduces and the distributed argmax
        m = native_model_tp(c, sd, "fp32", rank, world, nids[0], max_batch=8, max_tokens=80)
        out["fp32"] = [m.decode_step([int(t)], [p])[0][0] for p, t in enumerate(toks)]
        m.close()
        # bf16: tensor-core prefill of 2 prompts, then a batch-6 tensor-core decode step
        m = native_model_tp(c, sd, "bf16", rank, world, nids[1], max_batch=8, max_tokens=80)
        prompts = np.random.default_rng(52).integers(0, c["vocab"], (2, 30)).astype(np.int32)
        out["prefill"] = m.prefill(prompts)[0]
        seqs = np.random.default_rng(53).integers(0, c["vocab"], (6, 5))
        last = None
        for p in range(5):
            last = m.decode_step(seqs[:, p].tolist(), [p] * 6, slots=[2, 3, 4, 5, 6, 7])[0]
        out["batch6"] = last
        m.close()
        q.put((rank, out, None))
    except Exception as e:  # report instead of hanging the parent
        import traceback
        q.put((rank, None, traceback.format_exc()))
