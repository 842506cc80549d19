"""One tensor-parallel rank of the GPU TP tests (run in a spawned process per GPU).  Every model gets its
own NCCL unique id: an id bootstraps exactly one communicator."""
import numpy as np


def parity_fixture():
    """The model and the oracle's answers of tests/golden/tp_parity.npz (made by make_tp_parity.py): the
    library's synthetic weights at a geometry whose tp-2 shard runs the persistent step kernel."""
    import os
    from tests.golden.make_tp_parity import GEOM
    fx = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tp_parity.npz"))
    return GEOM, fx


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
        # bf16 batch-1 greedy generation: the persistent step kernel with the cross-rank exchange over NVLink
        g, fx = parity_fixture()
        cfg = native.make_config(g["dim"], g["hidden_dim"], g["layers"], g["heads"], g["kv_heads"], g["head_dim"],
                                 g["vocab"], g["seq_len"], False, native.QKNORM_VECTOR, False, native.DTYPE_BF16,
                                 native.DTYPE_BF16, 1, 8, decode_kernels=2)
        m = native.NativeModel(cfg, rank, rank, world, nids[2])
        m.init_synthetic(int(fx["seed"]), float(fx["std"]))
        m.finalize()
        prompt = fx["prompt"].astype(np.int32)
        out["greedy"] = m.generate(prompt, 8 + 24)[0]
        out["step_launches"] = m.last_launch_count  # 1: the persistent step kernel ran
        # the same greedy steps replayed from a captured CUDA graph (token/position advance on the device)
        import torch
        torch.cuda.set_device(rank)
        m.reset()
        m.prefill(prompt[None], want_logits=False)
        m.reserve(0, 40)
        dt = torch.tensor([int(out["greedy"][8])], dtype=torch.int32, device="cuda")
        dp = torch.tensor([8], dtype=torch.int32, device="cuda")
        ds = torch.zeros(1, dtype=torch.int32, device="cuda")
        dam = torch.zeros(1, dtype=torch.int32, device="cuda")
        m.capture_decode(dt.data_ptr(), ds.data_ptr(), dp.data_ptr(), 1, 0, dam.data_ptr())
        graph = []
        for _ in range(23):
            m.replay_decode(1)
            m.synchronize()
            graph.append(int(dt.item()))
        out["graph"] = graph
        m.close()
        q.put((rank, out, None))
    except Exception as e:  # report instead of hanging the parent
        import traceback
        q.put((rank, None, traceback.format_exc()))
