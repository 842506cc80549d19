"""Benchmark: Qwen3-8B bf16 batch-1 greedy decode on B200 (tensor-parallel over --gpus N).

Workload: Qwen3-8B geometry (hidden 4096, 36 layers, 32 Q / 8 KV heads,
head_dim 128, intermediate 12288, vocab 151936, untied lm_head), random-init bf16 weights from
the library's seeded synthetic generator (N(0, 0.02)-shaped), a 512-token uniform-random prompt,
then greedy decode.  One step = one decode token of the batch through the whole model
(36 layers + lm_head + argmax), captured once as a CUDA graph and replayed.  Inputs are the
15 GB of weights, far larger than the 126 MB L2, so every step streams them from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

GEOM_8B = dict(dim=4096, hidden_dim=12288, layers=36, heads=32, kv_heads=8, head_dim=128, vocab=151936,
               shared_weights=0, qk_norm=1, has_qkv_bias=0, rope_theta=1e6, eps=1e-6)
PROMPT = 512  # default prompt length (--prompt-len)
METRIC = "Qwen3-8B decode tok/s (batch 1, bf16, 512-token prompt)"


def weight_bytes(g, tp=1, wsz=2):
    D, F, V = g["dim"], g["hidden_dim"], g["vocab"]
    Q, KV = g["heads"] * g["head_dim"], g["kv_heads"] * g["head_dim"]
    per_layer = (Q + 2 * KV) * D + D * Q + 2 * F * D + D * F
    return dict(qkv=(Q + 2 * KV) * D * wsz // tp, o_proj=D * Q * wsz // tp, gate_up=2 * F * D * wsz // tp,
                down=D * F * wsz // tp, lm_head=V * D * wsz // tp, layers_total=per_layer * g["layers"] * wsz // tp)


def kv_bytes_per_token(g, ctx, tp=1, esz=2):
    return g["layers"] * 2 * (g["kv_heads"] // tp) * g["head_dim"] * esz * ctx


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None

    def stop(self):
        if not self.p:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        out, _ = self.p.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def peaks_of():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return {}


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


# ----------------------------------------------------------------------------------- CPU arm
def cpu_sample(tokens: int, warmup_slices: int, threads: int | None = None):
    """The oracle port on the host cores: the 8B geometry in fp32 with one layer's weights shared by all
    36 layers (identical bytes streamed per layer, 34 GB less host memory), context 512.  One decode
    token = 36 layer slices, each followed by 1/36 of the lm_head rows; `tokens` whole tokens are timed.
    threads: OpenMP threads (default: every host core, whatever OMP_NUM_THREADS says)."""
    from oracle import oracle as O
    O.set_threads(threads or os.cpu_count() or 1)
    c = dict(GEOM_8B, seq_len=PROMPT + 64, share_layers=1)
    m = O.OracleModel(c, "f32")
    m.init_synthetic(0, 0.02)
    L, V = c["layers"], c["vocab"]
    rows = [(V * i) // L for i in range(L + 1)]
    for i in range(warmup_slices):
        m.bench_slice(i % L, PROMPT, rows[i % L], rows[i % L + 1])
    per_token = []
    for _ in range(tokens):
        t0 = time.perf_counter()
        for i in range(L):
            m.bench_slice(i, PROMPT, rows[i], rows[i + 1])
        per_token.append(time.perf_counter() - t0)
    m.close()
    dt = sum(per_token)
    return tokens / dt, dt, O.num_threads("f32")


def run_reference(args):
    """The reference arm: the Java reference cannot run on this image (no JDK), so its CPU path is the
    oracle port, on every host core, one whole decode token per step."""
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    tok_s, dt, cores = cpu_sample(args.steps, 36 * args.warmup)
    sample = (f"oracle port (fp32, OpenMP, {cores} threads) at the Qwen3-8B geometry, layer weights shared, "
              f"context {PROMPT}; {args.steps} whole decode tokens (36 layers + full lm_head each), "
              f"{dt:.1f} s")
    line = {"metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "qwen3-8b decode batch 1 (CPU sample)", "model": "Qwen3-8B", "global_batch": 1,
                       "seq_len": PROMPT, "parallelism": "cpu"},
            "impl": "reference",
            "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0



def prefill_flops(g, nseq, L):
    D, F = g["dim"], g["hidden_dim"]
    Q, KV = g["heads"] * g["head_dim"], g["kv_heads"] * g["head_dim"]
    linear = (Q + 2 * KV) * D + D * Q + 2 * F * D + D * F
    lin = 2.0 * linear * g["layers"] * nseq * L
    attn = 2.0 * L * L * g["head_dim"] * g["heads"] * g["layers"] * nseq  # causal QK^T + PV
    return lin + attn, lin, attn


def run_batched(args, rank, world, local, nid, peaks):
    """prefill of 8 x 4096 tokens on the tensor cores, then batch-64 decode at 4096
    context (the 64 sequences are prefilled in chunks of 32768 tokens first)."""
    import numpy as np
    import torch
    from common_b200 import native
    g = GEOM_8B
    NSEQ, L, B = args.prefill_seqs, args.prefill_len, args.decode_batch
    steps = args.batch_steps
    seq_len = L + 3 + steps + 8
    cfg = native.make_config(g["dim"], g["hidden_dim"], g["layers"], g["heads"], g["kv_heads"], g["head_dim"],
                             g["vocab"], seq_len, False, native.QKNORM_VECTOR, False, native.DTYPE_BF16,
                             native.DTYPE_BF16, B, NSEQ * L)
    m = native.NativeModel(cfg, local, rank, world, nid)
    m.init_synthetic(0, 0.02)
    m.finalize()
    stream = torch.cuda.ExternalStream(m.stream)
    rng = np.random.default_rng(1)
    prompts = rng.integers(0, g["vocab"], (B, L)).astype(np.int32)

    def sync_all():
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    # ---- prefill NSEQ x L (warm-up once, then timed repeats; each repeat rewrites the same slots) ----
    m.prefill(prompts[:NSEQ], want_logits=False)
    times = []
    for _ in range(args.prefill_reps):
        sync_all()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        m.prefill(prompts[:NSEQ], want_logits=False)
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    pms = min(times) if world == 1 else max(times)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([pms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pms = float(t.item())
    fl, lin, att = prefill_flops(g, NSEQ, L)
    tf = fl / (pms * 1e-3) / 1e12
    peak_tf = peaks.get("bf16_tflops", 1590.0)
    pd, pk = None, None
    prefill = {"tok_s": NSEQ * L / (pms * 1e-3), "ms": pms, "seqs": NSEQ, "seq_len": L, "flops": fl,
               "tflops": tf, "roofline": {"bound": "tensor", "achieved": tf / world, "peak": peak_tf, "unit": "TFLOP/s",
                                          "frac": tf / world / peak_tf, "per": "GPU",
                                          "peak_source": "MEASURED_PEAKS.json bf16_tflops (burst)" if peaks else "fallback",
                                          # the prefill runs for about half a second under the 1 kW power cap: the
                                          # seconds-long cuBLAS loop is the like-for-like denominator
                                          "peak_sustained": peaks.get("bf16_tflops_sustained"),
                                          "frac_sustained": (tf / world / peaks["bf16_tflops_sustained"]
                                                             if peaks.get("bf16_tflops_sustained") else None)},
               "flops_split": {"linear": lin, "attention_causal": att, "lm_head": "last position only"},
               "timing": "qw_prefill through the host API (tokens from host memory), CUDA events, best of "
                         f"{args.prefill_reps}" if world == 1 else "max over ranks"}

    # per-kernel split of one prefill (CUDA events around every launch)
    pk_ms, pk_kind = m.profile_prefill(prompts[:NSEQ])
    split = {}
    for x, kk in zip(pk_ms, pk_kind):
        split[native.KERNEL_NAMES[int(kk)]] = split.get(native.KERNEL_NAMES[int(kk)], 0.0) + float(x)
    prefill["kernel_ms"] = split
    if split.get("attn"):
        att_tf = att / world / (split["attn"] * 1e-3) / 1e12
        prefill["attention"] = {"kernel": "qw_flash_prefill_tc_kernel (tcgen05, TMEM, TMA)"
                                if os.environ.get("QW_TC_ATTN", "1") != "0" else "qw_flash_prefill_kernel (mma.sync)", "ms": split["attn"],
                                "flops": att / world, "tflops": att_tf, "frac": att_tf / peak_tf,
                                "flops_counted": "causal: 2 * 2 * L^2 / 2 * head_dim per head, layer and sequence"}
    # ---- batch-B decode at context L: prefill the remaining slots, capture, replay ----
    for c0 in range(NSEQ, B, NSEQ):
        m.prefill(prompts[c0:c0 + NSEQ], slots=np.arange(c0, min(B, c0 + NSEQ), dtype=np.int32), want_logits=False)
    for b in range(B):
        m.reserve(b, seq_len)
    dt = torch.tensor(rng.integers(0, g["vocab"], B), dtype=torch.int32, device="cuda")
    dp = torch.full((B,), L, dtype=torch.int32, device="cuda")
    ds = torch.arange(B, dtype=torch.int32, device="cuda")
    dam = torch.zeros(B, dtype=torch.int32, device="cuda")
    m.capture_decode(dt.data_ptr(), ds.data_ptr(), dp.data_ptr(), B, 0, dam.data_ptr())
    launches = m.last_launch_count
    m.replay_decode(3)
    sync_all()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    m.replay_decode(steps)
    e1.record(stream)
    torch.cuda.synchronize()
    dms = e0.elapsed_time(e1)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([dms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dms = float(t.item())
    ctx_mid = L + 3 + steps // 2
    step_bytes = sum(v for k, v in weight_bytes(g, world).items() if k in ("layers_total", "lm_head")) + \
        B * kv_bytes_per_token(g, ctx_mid, world)
    gbs = step_bytes / (dms / steps * 1e-3) / 1e9
    peak = peaks.get("hbm_gbs", 6650.0)
    # per-kernel split of one eager step
    m.set_device_inputs(dt.cpu().numpy(), dp.cpu().numpy())
    d, k = m.profile_decode(B)
    kern = {}
    for x, kk in zip(d, k):
        kern[native.KERNEL_NAMES[int(kk)]] = kern.get(native.KERNEL_NAMES[int(kk)], 0.0) + float(x)
    decode = {"tok_s": B * steps / (dms * 1e-3), "ms_per_step": dms / steps, "batch": B, "context": [L + 3, L + 3 + steps],
              "steps": steps, "launches_per_step": launches,
              "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                           "bytes_per_step": step_bytes, "per": "GPU" if world == 1 else "rank"},
              "kernel_ms_per_step": kern}
    m.close()
    return {"prefill": prefill, "decode_b%d" % B: decode}

# ----------------------------------------------------------------------------------- parity gate
# the model of tests/golden/make_tp_parity.py (2 layers, hidden 1024, 32 Q / 8 KV heads of 128, intermediate
# 4096, vocab 4096), whose oracle answers tests/golden/tp_parity.npz holds
PARITY_GEOM = dict(dim=1024, hidden_dim=4096, layers=2, heads=32, kv_heads=8, head_dim=128, vocab=4096, seq_len=64)


def parity_check(rank, world, local, share_id, decode_kernels=0):
    """Before anything is timed, at every GPU count: the tensor-parallel model over `world` ranks against the
    oracle's answers (committed fixture).  fp32 mode: logits at the 8 prompt positions within 1e-3 relative
    L2.  bf16 mode (the decode path the bench times): the oracle's 40 tokens fed one per step, every logits
    row within 2e-2 relative L2 and every greedy choice after the prompt identical; and the batched
    tensor-core path (batch 8) generating the same 32 greedy tokens in every sequence."""
    import numpy as np
    from common_b200 import native
    fx = np.load(os.path.join(ROOT, "tests", "golden", "tp_parity.npz"))
    g = PARITY_GEOM
    seed, std = int(fx["seed"]), float(fx["std"])

    def rel(a, b):
        a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
        return float(np.linalg.norm(a - b) / np.linalg.norm(b))

    out = {"fixture": "tests/golden/tp_parity.npz", "tp": world}
    for prec, dt in (("fp32", native.DTYPE_F32), ("bf16", native.DTYPE_BF16)):
        cfg = native.make_config(g["dim"], g["hidden_dim"], g["layers"], g["heads"], g["kv_heads"], g["head_dim"],
                                 g["vocab"], g["seq_len"], False, native.QKNORM_VECTOR, False, dt, dt, 1, 0,
                                 decode_kernels=decode_kernels if prec == "bf16" else 0)
        m = native.NativeModel(cfg, local, rank, world, share_id(native.unique_id))
        m.init_synthetic(seed, std)
        m.finalize()
        if prec == "fp32":
            errs = []
            for p, t in enumerate(fx["prompt"]):
                lg, _ = m.decode_step([int(t)], [p])
                errs.append(rel(lg[0], fx["fp32_logits"][p]))
            out["fp32_max_rel_l2"] = max(errs)
        else:
            toks, want = fx["bf16_tokens"], fx["bf16_logits"].astype(np.float32)
            errs, bad = [], []
            for p, t in enumerate(toks):
                lg, am = m.decode_step([int(t)], [p])
                errs.append(rel(lg[0], want[p]))
                if p + 1 < len(toks) and p + 1 >= len(fx["prompt"]) and int(am[0]) != int(toks[p + 1]):
                    bad.append(p + 1)
            out["bf16_max_rel_l2"] = max(errs)
            out["bf16_greedy_steps"] = len(toks) - len(fx["prompt"])
            out["bf16_token_mismatches"] = bad
            out["bf16_launches_per_token"] = m.last_launch_count
        m.close()
    # the batched tensor-core path (tcgen05 prefill of 8 copies of the prompt, then batch-8 greedy decode
    # through qw_generate): every sequence must produce the oracle's tokens
    cfg = native.make_config(g["dim"], g["hidden_dim"], g["layers"], g["heads"], g["kv_heads"], g["head_dim"],
                             g["vocab"], g["seq_len"], False, native.QKNORM_VECTOR, False, native.DTYPE_BF16,
                             native.DTYPE_BF16, 8, 64)
    m = native.NativeModel(cfg, local, rank, world, share_id(native.unique_id))
    m.init_synthetic(seed, std)
    m.finalize()
    toks = fx["bf16_tokens"]
    got = m.generate(np.repeat(fx["prompt"][None].astype(np.int32), 8, 0), len(toks))
    m.close()
    out["batched_b8_token_mismatches"] = sorted({int(p) for b in range(8) for p in np.nonzero(got[b] != toks)[0]})
    out["ok"] = bool(out["fp32_max_rel_l2"] < 1e-3 and out["bf16_max_rel_l2"] < 2e-2 and not out["bf16_token_mismatches"]
                     and not out["batched_b8_token_mismatches"])
    return out


# ----------------------------------------------------------------------------------- C2 / C5 decode legs
GEOM_1P7B = dict(dim=2048, hidden_dim=6144, layers=28, heads=16, kv_heads=8, head_dim=128, vocab=151936,
                 shared_weights=1, qk_norm=1, has_qkv_bias=0, rope_theta=1e6, eps=1e-6)
GEOM_32B = dict(dim=5120, hidden_dim=25600, layers=64, heads=64, kv_heads=8, head_dim=128, vocab=151936,
                shared_weights=0, qk_norm=1, has_qkv_bias=0, rope_theta=1e6, eps=1e-6)


def run_decode_config(name, g, B, prompt_len, gen, rank, world, local, nid, peaks, chunk_tokens=32768):
    """A batched greedy decode configuration: B sequences of uniform-random prompts prefilled on the tensor
    cores (chunks of chunk_tokens), then `gen` batch-B decode steps captured as one CUDA graph step and
    replayed (device-resident token feedback); tok/s = B * gen / the replay time (CUDA events, max over
    ranks).  Roofline: HBM, bytes per step = every weight byte of the rank + the KV rows read."""
    import numpy as np
    import torch
    from common_b200 import native
    seq_len = prompt_len + gen + 8
    per_chunk = max(1, min(B, chunk_tokens // prompt_len))
    cfg = native.make_config(g["dim"], g["hidden_dim"], g["layers"], g["heads"], g["kv_heads"], g["head_dim"],
                             g["vocab"], seq_len, g["shared_weights"], native.QKNORM_VECTOR, False, native.DTYPE_BF16,
                             native.DTYPE_BF16, B, per_chunk * prompt_len)
    m = native.NativeModel(cfg, local, rank, world, nid)
    m.init_synthetic(0, 0.02)
    m.finalize()
    stream = torch.cuda.ExternalStream(m.stream)
    rng = np.random.default_rng(1)
    prompts = rng.integers(0, g["vocab"], (B, prompt_len)).astype(np.int32)
    first = np.zeros(B, np.int32)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for c0 in range(0, B, per_chunk):
        sl = np.arange(c0, min(B, c0 + per_chunk), dtype=np.int32)
        _, am = m.prefill(prompts[c0:c0 + per_chunk], slots=sl, want_logits=False)
        first[c0:c0 + len(sl)] = am
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    for b in range(B):
        m.reserve(b, seq_len)
    dt = torch.tensor(first, dtype=torch.int32, device="cuda")
    dp = torch.full((B,), prompt_len, dtype=torch.int32, device="cuda")
    ds = torch.arange(B, dtype=torch.int32, device="cuda")
    dam = torch.zeros(B, dtype=torch.int32, device="cuda")
    m.capture_decode(dt.data_ptr(), ds.data_ptr(), dp.data_ptr(), B, 0, dam.data_ptr())
    launches = m.last_launch_count
    warm = 3
    m.replay_decode(warm)
    m.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    m.replay_decode(gen - warm)
    e1.record(stream)
    torch.cuda.synchronize()
    m.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    steps = gen - warm
    ctx_mid = prompt_len + warm + steps // 2
    wb = weight_bytes(g, world)
    step_bytes = wb["layers_total"] + wb["lm_head"] + B * kv_bytes_per_token(g, ctx_mid, world)
    gbs = step_bytes / (ms / steps * 1e-3) / 1e9
    peak = peaks.get("hbm_gbs", 6650.0)
    # per-kernel split of one eager step (CUDA events around every launch)
    m.set_device_inputs(dt.cpu().numpy(), dp.cpu().numpy())
    kd, kk = m.profile_decode(B)
    kern = {}
    for x, k in zip(kd, kk):
        kern[native.KERNEL_NAMES[int(k)]] = kern.get(native.KERNEL_NAMES[int(k)], 0.0) + float(x)
    m.close()
    return {"kernel_ms_per_step": kern, "workload": name, "tok_s": B * steps / (ms * 1e-3), "ms_per_step": ms / steps, "batch": B,
            "prompt_len": prompt_len, "generated": gen, "timed_steps": steps, "warmup_steps": warm,
            "context": [prompt_len + warm, prompt_len + gen], "launches_per_step": launches, "parallelism": f"tp{world}",
            "prefill_s": prefill_s,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                         "bytes_per_step": step_bytes, "per": "GPU" if world == 1 else "rank"}}


# ----------------------------------------------------------------------------------- GPU arm
def run_ours(args):
    import numpy as np
    import torch
    from common_b200 import build, native

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    build.build()
    from common_b200 import parallel
    parity = None if args.no_parity else parity_check(rank, world, local, parallel.share_unique_id,
                                                          args.decode_kernels)
    if parity and not parity["ok"]:
        print(json.dumps({"parity_failed": parity}), file=sys.stderr, flush=True)
    nid = parallel.share_unique_id(native.unique_id)  # one NCCL id per communicator (per model)
    g = GEOM_8B
    B = 1
    e2e_steps = args.e2e_steps
    seq_len = PROMPT + args.warmup + args.steps + e2e_steps + 8
    cfg = native.make_config(g["dim"], g["hidden_dim"], g["layers"], g["heads"], g["kv_heads"], g["head_dim"],
                             g["vocab"], seq_len, False, native.QKNORM_VECTOR, False, native.DTYPE_BF16,
                             native.DTYPE_BF16, B, PROMPT,  # the prompt is one tensor-core prefill chunk
                             decode_kernels=args.decode_kernels)
    m = native.NativeModel(cfg, local, rank, world, nid)
    m.init_synthetic(0, 0.02)
    m.finalize()
    prompt = np.random.default_rng(1).integers(0, g["vocab"], PROMPT).astype(np.int32)
    _, first = m.prefill(prompt[None], want_logits=False)
    m.reserve(0, seq_len)
    dt = torch.tensor(first, dtype=torch.int32, device="cuda")
    dp = torch.tensor([PROMPT], dtype=torch.int32, device="cuda")
    ds = torch.zeros(B, dtype=torch.int32, device="cuda")
    dam = torch.zeros(B, dtype=torch.int32, device="cuda")
    m.capture_decode(dt.data_ptr(), ds.data_ptr(), dp.data_ptr(), B, 0, dam.data_ptr())
    launches_per_step = m.last_launch_count
    stream = torch.cuda.ExternalStream(m.stream)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    m.replay_decode(args.warmup)
    m.synchronize()  # raises if a bounded device-side wait gave up
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    m.replay_decode(args.steps)
    e1.record(stream)
    barrier()
    m.synchronize()
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ctx_mid = PROMPT + args.warmup + args.steps // 2
    value = args.steps * B / (ms / 1e3)

    # ---- per-kernel durations (CUDA events around every launch of one eager step) ----
    pos_now = int(dp.item())
    m.set_device_inputs([int(dt.item())], [pos_now])
    kinds_ms: dict[str, list] = {}
    for _ in range(3):
        d, k = m.profile_decode(B)
        for x, kk in zip(d, k):
            kinds_ms.setdefault(native.KERNEL_NAMES[int(kk)], []).append(float(x))
    avg = {k: sum(v) / len(v) for k, v in kinds_ms.items()}
    tot = {k: sum(v) / 3 for k, v in kinds_ms.items()}
    wb = weight_bytes(g, world)
    if "step" in avg:  # the persistent whole-step kernel: every weight byte + the KV read of one token
        dom, dom_name = "step", "step (persistent batch-1 decode step: all layers + lm_head + argmax)"
        dom_bytes = wb["layers_total"] + wb["lm_head"] + kv_bytes_per_token(g, pos_now + 1, world)
    else:
        dom, dom_name = "gate_up", "gemv gate_up (rmsnorm+SwiGLU)"
        dom_bytes = wb[dom]
    achieved = dom_bytes / (avg[dom] * 1e-3) / 1e9
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    peak = peaks.get("hbm_gbs", 6650.0)
    traffic = None
    try:
        traffic = json.load(open(os.path.join(ROOT, "profiles", "decode_traffic.json")))[dom]
    except Exception:
        pass
    step_bytes = wb["layers_total"] + wb["lm_head"] + kv_bytes_per_token(g, ctx_mid, world)
    step_gbs = step_bytes / (ms / args.steps * 1e-3) / 1e9

    # ---- end to end through the public host API: token in (pinned H2D), argmax out (D2H) ----
    e2e = None
    if e2e_steps:
        tok = int(dt.item())
        pos = int(dp.item())
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for i in range(e2e_steps):
            _, am = m.decode_step([tok], [pos + i], want_logits=False)
            tok = int(am[0])
        s1.record(stream)
        barrier()
        ems = s0.elapsed_time(s1)
        if world > 1:
            t = torch.tensor([ems], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        e2e = {"value": e2e_steps * B / (ems / 1e3), "unit": "tok/s", "h2d_bytes_per_step": 12 * B,
               "d2h_bytes_per_step": 4 * B, "steps": e2e_steps,
               "api": "qw_decode_step (host token/position/slot in, host argmax out)"}

    m.close()
    torch.cuda.empty_cache()
    extra = {}
    if world == 1 and not args.no_configs:
        extra["c2_decode_b16"] = run_decode_config(
            "qwen3-1.7b batch-16 decode, 2048-token prompts, 128 generated (BASELINE configs[1])", GEOM_1P7B, 16, 2048,
            128, rank, world, local, None, peaks_of())
        torch.cuda.empty_cache()
    if world == 8 and not args.no_configs:
        extra["c5_decode_b64"] = run_decode_config(
            "qwen3-32b tp8 batch-64 decode, paged KV at 8192 context, 128 generated (BASELINE configs[4])", GEOM_32B,
            64, 8192, 128, rank, world, local, parallel.share_unique_id(native.unique_id), peaks_of())
        torch.cuda.empty_cache()
    batched = None
    if not args.no_batched:
        batched = run_batched(args, rank, world, local, parallel.share_unique_id(native.unique_id), peaks)
        torch.cuda.empty_cache()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tok_s, dts, cores = cpu_sample(args.cpu_tokens, 2)
        cpu = {"value": tok_s, "unit": "tok/s", "cores": cores, "kind": "port",
               "sample": f"oracle port fp32 at the 8B geometry (layer weights shared), {args.cpu_tokens} whole decode "
                         f"tokens (36 layers + full lm_head) at context {PROMPT}, {dts:.1f} s"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": "qwen3-8b decode batch 1 (BASELINE configs[2])", "model": "Qwen3-8B",
                           "global_batch": B, "seq_len": PROMPT, "context_range": [PROMPT + args.warmup,
                                                                                   PROMPT + args.warmup + args.steps],
                           "parallelism": f"tp{world}", "l2": "weights 15 GB >> 126 MB L2 (no flush needed)",
                           "timing": "CUDA graph replay, CUDA events on the model stream, max over ranks"},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "traffic": traffic, "kernel": dom_name,
                             "bytes_per_launch": dom_bytes, "launch_ms": avg[dom],
                             "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks else "fallback 6650 GB/s",
                             "step_gbs": step_gbs, "step_frac": step_gbs / peak},
                "kernel_ms_per_step": tot, "gpu_launches": launches_per_step * args.steps,
                "launches_per_step": launches_per_step, "clocks": clk, "e2e": e2e, "cpu_baseline": cpu}
        line["parity"] = parity
        if batched:
            line.update(batched)
        line.update(extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_case(args):
    """Small fixed workloads for profiler captures (a few GB on the device, few launches):
      step-small  the 8B geometry cut to --layers layers, 4 batch-1 decode steps (the persistent step kernel)
      gemm        one qw_op_linear GEMM (--gemm M K T EPI) timed with CUDA events
      attn-b64    the 8B geometry cut to 2 layers, --decode-batch (64) sequences prefilled to 2048 tokens, 3 batched
                  decode steps
      prefill-small  the 8B geometry cut to 2 layers, two prefills of 8 x 4096 tokens
    """
    import numpy as np
    from common_b200 import build, native
    build.build()
    g = GEOM_8B
    if args.case == "gemm":
        import torch
        M, K, T, epi = args.gemm
        W = (torch.randn(M, K, device="cuda") * 0.02).bfloat16()
        X = torch.randn(T, K, device="cuda").bfloat16()
        out = torch.zeros(T, M // 2 if epi == 2 else M, device="cuda",
                          dtype=torch.bfloat16 if epi == 2 else torch.float32)

        def once():
            native.op_linear(W.data_ptr(), M, K, X.data_ptr(), T, epi, 0, out.data_ptr() if epi == 1 else 0,
                             out.data_ptr())
        for _ in range(3):
            once()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            once()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / 10
        print(json.dumps({"case": "gemm", "M": M, "K": K, "T": T, "epi": epi, "ms": ms,
                          "tflops": 2.0 * M * K * T / ms / 1e9}))
        return 0
    if args.case == "prefill-small":
        # the 8B geometry cut to 2 layers, one prefill of 8 x 4096 tokens (tcgen05 GEMMs + tcgen05 attention)
        cfg = native.make_config(g["dim"], g["hidden_dim"], 2, g["heads"], g["kv_heads"], g["head_dim"], g["vocab"],
                                 4096 + 16, False, native.QKNORM_VECTOR, False, native.DTYPE_BF16, native.DTYPE_BF16,
                                 8, 32768)
        m = native.NativeModel(cfg, 0)
        m.init_synthetic(0, 0.02)
        m.finalize()
        prompts = np.random.default_rng(1).integers(0, g["vocab"], (8, 4096)).astype(np.int32)
        for _ in range(2):
            m.prefill(prompts, want_logits=False)
        m.synchronize()
        m.close()
        print(json.dumps({"case": args.case, "ok": True}))
        return 0
    layers = args.layers if args.case == "step-small" else 2
    B, L = (1, 1024) if args.case == "step-small" else (args.decode_batch, 2048)
    cfg = native.make_config(g["dim"], g["hidden_dim"], layers, g["heads"], g["kv_heads"], g["head_dim"], g["vocab"],
                             L + 16, False, native.QKNORM_VECTOR, False, native.DTYPE_BF16, native.DTYPE_BF16, B,
                             16384 if B > 1 else 0)
    m = native.NativeModel(cfg, 0)
    m.init_synthetic(0, 0.02)
    m.finalize()
    if args.case == "step-small":
        for p in range(4):
            m.decode_step([5], [p], want_logits=False)
    else:
        prompts = np.random.default_rng(1).integers(0, g["vocab"], (B, L)).astype(np.int32)
        for c0 in range(0, B, 8):
            m.prefill(prompts[c0:c0 + 8], slots=np.arange(c0, c0 + 8, dtype=np.int32), want_logits=False)
        toks = np.random.default_rng(2).integers(0, g["vocab"], B)
        for st in range(3):
            m.decode_step(toks.tolist(), [L + st] * B, want_logits=False)
    m.synchronize()
    m.close()
    print(json.dumps({"case": args.case, "ok": True}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=240)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=64)
    ap.add_argument("--cpu-tokens", type=int, default=30, help="whole tokens of the CPU baseline leg")
    ap.add_argument("--no-batched", action="store_true", help="skip the prefill / batch-64 decode measurements")
    ap.add_argument("--prefill-seqs", type=int, default=8)
    ap.add_argument("--prefill-len", type=int, default=4096)
    ap.add_argument("--prefill-reps", type=int, default=3)
    ap.add_argument("--decode-batch", type=int, default=64)
    ap.add_argument("--batch-steps", type=int, default=32)
    ap.add_argument("--case", choices=["step-small", "gemm", "attn-b64", "prefill-small"], help="a small profiler workload instead")
    ap.add_argument("--layers", type=int, default=4, help="--case step-small: layers of the cut 8B model")
    ap.add_argument("--gemm", type=int, nargs=4, default=[24576, 4096, 4096, 2], metavar=("M", "K", "T", "EPI"))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the parity gate (profiler runs only)")
    ap.add_argument("--no-configs", action="store_true", help="skip the configs[1] (1 GPU) / configs[4] (8 GPUs) legs")
    ap.add_argument("--decode-kernels", type=int, default=0,
                    help="batch-1 decode path: 0 auto, 1 one kernel per operation, 2 the persistent step kernel")
    ap.add_argument("--prompt-len", type=int, default=PROMPT, help="shorter prompts for profiler runs")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    globals()["PROMPT"] = args.prompt_len
    if args.case:
        return run_case(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
