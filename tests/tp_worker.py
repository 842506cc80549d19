"""One tensor-parallel rank of the GPU TP tests (run in a spawned process per GPU).  Every model gets its
own NCCL unique id: an id bootstraps exactly one communicator."""
import numpy as np


def step_cfg():
    """A geometry the persistent step kernel runs at tp 2: dim, local q width and intermediate multiples of 512."""
    from tests.helpers import cfg_dict, state_dict
    c = cfg_dict(dim=1024, hidden_dim=2048, layers=2, heads=8, kv_heads=2, head_dim=128, vocab=2000, seq_len=64)
    return c, state_dict(c, seed=54, std=0.05, norm_noise=0.1)


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
        c, sd = step_cfg()
        m = native_model_tp(c, sd, "bf16", rank, world, nids[2], max_batch=1, max_tokens=8, decode_kernels=2)
        out["greedy"] = m.generate(np.array([3, 1, 4, 1, 5, 9, 2, 6], np.int32), 8 + 24)[0]
        out["step_launches"] = m.last_launch_count  # 1: the persistent step kernel ran
        # the same greedy steps replayed from a captured CUDA graph (token/position advance on the device)
        import torch
        torch.cuda.set_device(rank)
        m.reset()
        m.prefill(np.array([[3, 1, 4, 1, 5, 9, 2, 6]], np.int32), want_logits=False)
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
