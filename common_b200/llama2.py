"""Llama2 on the same transformer path (the reference's engine/ml/src/main/java/org/almostrealism/ml/llama2/Llama2.java).

The reference builds Llama2 from the unified transformer layer (AttentionFeatures.transformer with heads = kvHeads,
no QK-norm, no biases, rmsnorm epsilon 1e-5, AttentionFeatures.java:1607-1620) over a llama2.c checkpoint:
a little-endian header of seven int32 (dim, hidden_dim, layers, heads, kv_heads, vocab -- negative for an
untied classifier --, seq_len; TransformerConfig.java:69-80) followed by fp32 tensors in the order of
Llama2Weights.java:91-115 (embedding, attention rmsnorm, wq, wk, wv, wo, FFN rmsnorm, w1, w2, w3, final rmsnorm,
RoPE table as cos then sin planes, classifier when untied).  This module reads that file into the library's
state-dict keys and runs it through libqwen3_b200 (tokenisation is out of scope: token ids in, token ids out).
"""
from __future__ import annotations

import numpy as np

from . import native
from .qwen3 import Qwen3Config, StateDictionary

BOS_TOKEN = 1  # Llama2.run feeds BOS first


def read_checkpoint(path: str):
    """(Qwen3Config, StateDictionary) of a llama2.c checkpoint, in the reference's reading order."""
    raw = np.fromfile(path, dtype=np.uint8)
    head = raw[:28].view("<i4")
    dim, hidden, layers, heads, kv_heads, vocab, seq_len = (int(x) for x in head)
    shared = vocab > 0
    vocab = abs(vocab)
    if kv_heads != heads:
        # the reference passes headCount for both and reads wk / wv as (dim, dim)
        raise ValueError("Llama2 checkpoints with kv_heads != heads are not read by the reference either")
    hs = dim // heads
    f = raw[28:].view("<f4")
    off = 0

    def take(*shape):
        nonlocal off
        n = int(np.prod(shape))
        if off + n > f.size:
            raise ValueError("checkpoint is truncated")
        out = f[off:off + n].reshape(shape)
        off += n
        return out

    emb = take(vocab, dim)
    rms_att = take(layers, dim)
    wq, wk, wv, wo = take(layers, dim, dim), take(layers, dim, dim), take(layers, dim, dim), take(layers, dim, dim)
    rms_ffn = take(layers, dim)
    w1, w2, w3 = take(layers, hidden, dim), take(layers, dim, hidden), take(layers, hidden, dim)
    rms_final = take(dim)
    fre, fim = take(seq_len, hs // 2), take(seq_len, hs // 2)
    wcls = None if shared else take(vocab, dim)
    sd = {"model.embed_tokens.weight": emb, "model.norm.weight": rms_final,
          "rope.freq_cis": np.stack([fre, fim], -1).astype(np.float32)}
    if wcls is not None:
        sd["lm_head.weight"] = wcls
    for l in range(layers):
        p = f"model.layers.{l}."
        sd[p + "input_layernorm.weight"] = rms_att[l]
        sd[p + "post_attention_layernorm.weight"] = rms_ffn[l]
        sd[p + "self_attn.q_proj.weight"] = wq[l]
        sd[p + "self_attn.k_proj.weight"] = wk[l]
        sd[p + "self_attn.v_proj.weight"] = wv[l]
        sd[p + "self_attn.o_proj.weight"] = wo[l]
        sd[p + "mlp.gate_proj.weight"] = w1[l]
        sd[p + "mlp.down_proj.weight"] = w2[l]
        sd[p + "mlp.up_proj.weight"] = w3[l]
    cfg = Qwen3Config(dim, hidden, layers, heads, heads, vocab, seq_len, shared, ropeTheta=1e4, headSize=hs,
                      qkNorm=native.QKNORM_NONE)
    return cfg, StateDictionary(sd)


def write_checkpoint(path: str, cfg: Qwen3Config, sd: dict) -> None:
    """The inverse of read_checkpoint (for tests and conversions)."""
    vocab = cfg.vocabSize if cfg.sharedWeights else -cfg.vocabSize
    head = np.array([cfg.dim, cfg.hiddenDim, cfg.layerCount, cfg.headCount, cfg.kvHeadCount, vocab, cfg.seqLen],
                    "<i4")
    L = cfg.layerCount
    parts = [sd["model.embed_tokens.weight"]]
    parts += [np.stack([sd[f"model.layers.{l}.input_layernorm.weight"] for l in range(L)])]
    for k in ("q_proj", "k_proj", "v_proj", "o_proj"):
        parts += [np.stack([sd[f"model.layers.{l}.self_attn.{k}.weight"] for l in range(L)])]
    parts += [np.stack([sd[f"model.layers.{l}.post_attention_layernorm.weight"] for l in range(L)])]
    for k in ("gate_proj", "down_proj", "up_proj"):
        parts += [np.stack([sd[f"model.layers.{l}.mlp.{k}.weight"] for l in range(L)])]
    parts += [sd["model.norm.weight"], sd["rope.freq_cis"][..., 0], sd["rope.freq_cis"][..., 1]]
    if not cfg.sharedWeights:
        parts += [sd["lm_head.weight"]]
    with open(path, "wb") as fh:
        fh.write(head.tobytes())
        for p in parts:
            fh.write(np.ascontiguousarray(p, "<f4").tobytes())


class Llama2:
    """Llama2(checkpoint) with the reference's generation contract (Llama2.run: BOS at position 0, then the
    prompt, then sampled / greedy tokens), on libqwen3_b200."""

    def __init__(self, checkpoint: str, precision: str = "fp32", device: int = 0):
        from .qwen3 import Qwen3
        self.config, self.weights = read_checkpoint(checkpoint)
        self.model = Qwen3(self.config, self.weights, precision=precision, device=device, eps=1e-5)

    def setTemperature(self, t: float, seed: int | None = None):
        self.model.setTemperature(t, seed)

    def generate(self, prompt_tokens, steps: int) -> np.ndarray:
        toks = np.concatenate([[BOS_TOKEN], np.asarray(prompt_tokens, np.int32)]).astype(np.int32)
        return self.model.generate(toks, steps)

    def close(self):
        self.model.close()
