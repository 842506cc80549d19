"""Shared helpers for the GPU parity tests: identical weights into the CUDA library and the oracle."""
import numpy as np

from common_b200 import native
from oracle import oracle as O


def cfg_dict(dim=256, hidden_dim=512, layers=2, heads=4, kv_heads=2, head_dim=64, vocab=1000, seq_len=80,
             shared_weights=0, qk_norm=1, has_qkv_bias=0, rope_theta=1e6, eps=1e-6):
    return dict(dim=dim, hidden_dim=hidden_dim, layers=layers, heads=heads, kv_heads=kv_heads, head_dim=head_dim,
                vocab=vocab, seq_len=seq_len, shared_weights=shared_weights, qk_norm=qk_norm,
                has_qkv_bias=has_qkv_bias, rope_theta=rope_theta, eps=eps)


def state_dict(c, seed=0, std=0.02, norm_noise=0.0):
    """numpy default_rng(seed) N(0, std) weights; norm weights 1 (+ optional noise)."""
    rng = np.random.default_rng(seed)
    D, Q, KV, F, V = c["dim"], c["heads"] * c["head_dim"], c["kv_heads"] * c["head_dim"], c["hidden_dim"], c["vocab"]

    def n(*s):
        return rng.standard_normal(s, dtype=np.float32) * np.float32(std)

    def ones(*s):
        o = np.ones(s, np.float32)
        if norm_noise:
            o += rng.standard_normal(s, dtype=np.float32) * np.float32(norm_noise)
        return o

    sd = {"model.embed_tokens.weight": n(V, D), "model.norm.weight": ones(D)}
    if not c["shared_weights"]:
        sd["lm_head.weight"] = n(V, D)
    for l in range(c["layers"]):
        p = f"model.layers.{l}."
        sd[p + "input_layernorm.weight"] = ones(D)
        sd[p + "post_attention_layernorm.weight"] = ones(D)
        sd[p + "self_attn.q_proj.weight"] = n(Q, D)
        sd[p + "self_attn.k_proj.weight"] = n(KV, D)
        sd[p + "self_attn.v_proj.weight"] = n(KV, D)
        sd[p + "self_attn.o_proj.weight"] = n(D, Q)
        if c["has_qkv_bias"]:
            sd[p + "self_attn.q_proj.bias"] = n(Q)
            sd[p + "self_attn.k_proj.bias"] = n(KV)
            sd[p + "self_attn.v_proj.bias"] = n(KV)
        if c["qk_norm"]:
            sd[p + "self_attn.q_norm.weight"] = ones(c["heads"], c["head_dim"])
            sd[p + "self_attn.k_norm.weight"] = ones(c["kv_heads"], c["head_dim"])
        sd[p + "mlp.gate_proj.weight"] = n(F, D)
        sd[p + "mlp.up_proj.weight"] = n(F, D)
        sd[p + "mlp.down_proj.weight"] = n(D, F)
    return sd


def native_model(c, sd=None, precision="fp32", kv=None, max_batch=1, max_tokens=0, page_size=64, num_pages=0,
                 synthetic_seed=None, device=0, decode_kernels=0):
    dt = {"fp32": native.DTYPE_F32, "bf16": native.DTYPE_BF16}
    cfg = native.make_config(c["dim"], c["hidden_dim"], c["layers"], c["heads"], c["kv_heads"], c["head_dim"],
                             c["vocab"], c["seq_len"], c["shared_weights"], c["qk_norm"], c["has_qkv_bias"],
                             dt[precision], dt[kv or precision], max_batch, max_tokens, page_size, num_pages,
                             c["rope_theta"], c["eps"], decode_kernels)
    m = native.NativeModel(cfg, device)
    if sd is not None:
        for k, v in sd.items():
            m.load_tensor(k, v)
    else:
        m.init_synthetic(synthetic_seed, 0.02)
    m.finalize()
    return m


def oracle_model(c, sd=None, precision="f64", bf16_weights=False, synthetic_seed=None):
    o = O.OracleModel(c, precision)
    if sd is not None:
        o.load_state_dict(sd)
    else:
        o.init_synthetic(synthetic_seed, 0.02)
    if bf16_weights:
        o.round_weights_bf16()
    return o


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def native_model_tp(c, sd, precision, rank, world, nid, max_batch=1, max_tokens=0, page_size=64, decode_kernels=0):
    """One tensor-parallel rank (device = rank) holding its shard of the state dict."""
    dt = {"fp32": native.DTYPE_F32, "bf16": native.DTYPE_BF16}
    cfg = native.make_config(c["dim"], c["hidden_dim"], c["layers"], c["heads"], c["kv_heads"], c["head_dim"],
                             c["vocab"], c["seq_len"], c["shared_weights"], c["qk_norm"], c["has_qkv_bias"],
                             dt[precision], dt[precision], max_batch, max_tokens, page_size, 0,
                             c["rope_theta"], c["eps"], decode_kernels)
    m = native.NativeModel(cfg, rank, rank, world, nid)
    for k, v in sd.items():
        m.load_tensor(k, v)
    m.finalize()
    return m
