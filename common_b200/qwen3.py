"""Host-side mirror of the reference's Qwen3 runtime API, backed by libqwen3_b200.

Names, argument meaning and error behaviour follow engine/ml:
  Qwen3Config          engine/ml/src/main/java/org/almostrealism/ml/qwen3/Qwen3Config.java:574-588
  StateDictionary      engine/ml/src/main/java/org/almostrealism/ml/StateDictionary.java:70-160
  Qwen3                engine/ml/src/main/java/org/almostrealism/ml/qwen3/Qwen3.java:249-319 (constructor, getters)
  CompiledModel        domain/graph/src/main/java/org/almostrealism/model/CompiledModel.java:189-220 (forward, reset)
  AutoregressiveModel  engine/ml/src/main/java/org/almostrealism/ml/AutoregressiveModel.java:203-308, 405-434
Every call goes through the C ABI; there is no Python or CPU implementation of the math here.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np

from . import collections_pb, native

BOS_TOKEN = 151643  # Qwen3Tokenizer.java:76
EOS_TOKEN = 151645  # Qwen3Tokenizer.java:79


@dataclass
class Qwen3Config:
    """Model geometry.  headSize defaults to dim // headCount like TransformerConfig.java:104;
    pass it explicitly for Qwen3 geometries where heads*head_dim != dim."""
    dim: int
    hiddenDim: int
    layerCount: int
    headCount: int
    kvHeadCount: int
    vocabSize: int
    seqLen: int = 131072
    sharedWeights: bool = True
    ropeTheta: float = 1e6
    headSize: int | None = None
    qkNorm: int = native.QKNORM_VECTOR
    hasQkvBias: bool = False

    def __post_init__(self):
        if self.headSize is None:
            self.headSize = self.dim // self.headCount
        if self.headCount % self.kvHeadCount:
            raise ValueError("headCount must be a multiple of kvHeadCount")

    @property
    def kvDim(self) -> int:
        return self.kvHeadCount * self.headSize

    @property
    def qDim(self) -> int:
        return self.headCount * self.headSize


class StateDictionary:
    """Weights by HF key: StateDictionary(weights) over numpy arrays (float32, float64 or raw-bf16 uint16),
    or StateDictionary(weightsDirectory) over the reference's protobuf files (a directory, or one file),
    whose tensors are decoded when asked for (StateDictionary.java:63-150).  A model built from a
    directory-backed dictionary loads the files through the library (qw_load_state_dict_pb)."""

    def __init__(self, weights):
        if isinstance(weights, (str, os.PathLike)):
            self.weightsDirectory = os.fspath(weights)
            self._lazy = collections_pb.read_directory(self.weightsDirectory)
            self._w = {}
        else:
            self.weightsDirectory = None
            self._lazy = {}
            self._w = dict(weights)

    def get(self, key: str):
        if key not in self._w and key in self._lazy:
            self._w[key] = self._lazy[key].numpy()
        return self._w.get(key)

    def shape(self, key: str):
        """The tensor's shape without decoding it (None when absent)."""
        if key in self._lazy:
            return self._lazy[key].shape
        v = self._w.get(key)
        return None if v is None else tuple(v.shape)

    def containsKey(self, key: str) -> bool:
        return key in self._w or key in self._lazy

    def keySet(self):
        return (self._lazy.keys() | self._w.keys()) if self._lazy else self._w.keys()

    def items(self):
        return ((k, self.get(k)) for k in self.keySet())

    def save(self, path: str, precision: str = "fp32"):
        """StateDictionary.save(weights, path, precision) (StateDictionary.java:215-235)."""
        collections_pb.save({k: self.get(k) for k in self.keySet()}, path, precision)


def infer_config(sd: StateDictionary, headSize: int | None = None) -> Qwen3Config:
    """Qwen3.inferConfig equivalent (Qwen3.java:200-240): geometry from tensor shapes."""
    vocab, dim = sd.shape("model.embed_tokens.weight")
    layers = 0
    while sd.containsKey(f"model.layers.{layers}.input_layernorm.weight"):
        layers += 1
    hidden = sd.shape("model.layers.0.mlp.gate_proj.weight")[0]
    q_rows = sd.shape("model.layers.0.self_attn.q_proj.weight")[0]
    kv_rows = sd.shape("model.layers.0.self_attn.k_proj.weight")[0]
    qn = sd.shape("model.layers.0.self_attn.q_norm.weight")
    if headSize is None:
        headSize = qn[-1] if qn is not None and len(qn) == 2 else 128
    # identity of the two arrays, as Qwen3.java:230-231 compares references (never true for decoded files)
    shared = not sd.containsKey("lm_head.weight") or (
        sd.weightsDirectory is None and sd.get("lm_head.weight") is sd.get("model.embed_tokens.weight"))
    return Qwen3Config(dim, hidden, layers, q_rows // headSize, kv_rows // headSize, vocab, 131072, shared, 1e6,
                       headSize=headSize, qkNorm=native.QKNORM_VECTOR if qn is not None else native.QKNORM_NONE,
                       hasQkvBias=sd.containsKey("model.layers.0.self_attn.q_proj.bias"))


def synthetic_state_dict(cfg: Qwen3Config, seed: int = 0, std: float = 0.02) -> StateDictionary:
    """Random-init weights N(0, std) from numpy default_rng(seed), norm weights 1 (fp32)."""
    rng = np.random.default_rng(seed)
    D, Q, KV, F, V = cfg.dim, cfg.qDim, cfg.kvDim, cfg.hiddenDim, cfg.vocabSize

    def n(*shape):
        return rng.standard_normal(shape, dtype=np.float32) * np.float32(std)

    w = {"model.embed_tokens.weight": n(V, D), "model.norm.weight": np.ones(D, np.float32)}
    for l in range(cfg.layerCount):
        p = f"model.layers.{l}."
        w[p + "input_layernorm.weight"] = np.ones(D, np.float32)
        w[p + "post_attention_layernorm.weight"] = np.ones(D, np.float32)
        w[p + "self_attn.q_proj.weight"] = n(Q, D)
        w[p + "self_attn.k_proj.weight"] = n(KV, D)
        w[p + "self_attn.v_proj.weight"] = n(KV, D)
        w[p + "self_attn.o_proj.weight"] = n(D, Q)
        if cfg.hasQkvBias:
            w[p + "self_attn.q_proj.bias"] = n(Q)
            w[p + "self_attn.k_proj.bias"] = n(KV)
            w[p + "self_attn.v_proj.bias"] = n(KV)
        if cfg.qkNorm != native.QKNORM_NONE:
            w[p + "self_attn.q_norm.weight"] = np.ones((cfg.headCount, cfg.headSize), np.float32)
            w[p + "self_attn.k_norm.weight"] = np.ones((cfg.kvHeadCount, cfg.headSize), np.float32)
        w[p + "mlp.gate_proj.weight"] = n(F, D)
        w[p + "mlp.up_proj.weight"] = n(F, D)
        w[p + "mlp.down_proj.weight"] = n(D, F)
    if not cfg.sharedWeights:
        w["lm_head.weight"] = n(V, D)
    return StateDictionary(w)


def native_config(cfg: Qwen3Config, precision: str = "bf16", kv_precision: str | None = None, max_batch: int = 1,
                  max_tokens: int = 0, page_size: int = 64, eps: float = 1e-6) -> native.QwConfig:
    dt = {"bf16": native.DTYPE_BF16, "fp32": native.DTYPE_F32}
    kv = kv_precision or precision
    return native.make_config(cfg.dim, cfg.hiddenDim, cfg.layerCount, cfg.headCount, cfg.kvHeadCount, cfg.headSize,
                              cfg.vocabSize, cfg.seqLen, cfg.sharedWeights, cfg.qkNorm, cfg.hasQkvBias, dt[precision],
                              dt[kv], max_batch, max_tokens, page_size, 0, cfg.ropeTheta, eps)


class CompiledModel:
    """forward((1, dim) embedding row) -> (1, vocab) logits at the model's current position."""

    def __init__(self, owner: "Qwen3"):
        self._o = owner
        self.last_argmax = None

    def getInputShape(self):
        return (1, self._o.config.dim)

    def getOutputShape(self):
        return (1, self._o.config.vocabSize)

    def forward(self, x) -> np.ndarray:
        x = np.asarray(x, np.float32).reshape(1, self._o.config.dim)
        pos = int(self._o.position[0])
        logits, am = self._o.native.forward_hidden(x, [pos])
        self.last_argmax = int(am[0])
        return logits

    def reset(self):
        self._o.native.reset(-1)


class AutoregressiveModel:
    """The generation loop of AutoregressiveModel.next() (AutoregressiveModel.java:295-308): prompt tokens are
    fed first, then each step samples from the previous step's output -- greedily at temperature 0, else with
    the sampler Qwen3 builds in AutoregressiveModel.of (:405-434), drawn on the device."""

    def __init__(self, owner: "Qwen3"):
        self._o = owner
        self.currentStep = 0
        self.currentToken = BOS_TOKEN
        self.prompt = None
        self.promptLength = 0
        self.temperature = 0.0
        self._next_token = None

    def reset(self):
        self._o.native.reset(-1)
        self.currentStep = 0
        self._o.position[0] = 0
        self._next_token = None

    def setCurrentToken(self, t: int):
        self.currentToken = int(t)

    def setPrompt(self, prompt, length: int):
        self.prompt = None if prompt is None else [int(t) for t in prompt]
        self.promptLength = int(length)

    def getCurrentStep(self) -> int:
        return self.currentStep

    def setTemperature(self, t: float, seed: int | None = None):
        """AutoregressiveModel.setTemperature (:59-61).  The reference draws from an unseeded java.util.Random;
        here the draws come from java.util.Random(seed) on the device (seed from the clock when None)."""
        if t < 0:
            raise ValueError("temperature must be >= 0")
        if seed is None:
            import time
            seed = time.time_ns() & 0x7FFFFFFFFFFFFFFF
        self._o.native.set_sampling(float(t), 1.0, int(seed), 0)
        self.temperature = float(t)

    def next(self) -> int:
        if self.currentStep < self.promptLength:
            tok = self.prompt[self.currentStep]
        else:
            if self._next_token is None:
                raise RuntimeError("no previous output to sample from")
            tok = self._next_token
        if self.currentStep < self.promptLength - 1:
            # inside the prompt the output is not sampled (the reference draws only once the prompt is fed)
            _, am = self._o.native.decode_step([tok], [self.currentStep], want_logits=False)
            self._next_token = int(am[0])
        else:
            self._next_token = int(self._o.native.decode_sample([tok], [self.currentStep])[0])
        self.currentToken = tok
        self.currentStep += 1
        self._o.position[0] = self.currentStep
        return tok


class Qwen3:
    """Qwen3(config, stateDict[, tokenizer]) on one B200 (or one TP rank)."""

    def __init__(self, config: Qwen3Config, stateDict: StateDictionary | None, tokenizer=None, *,
                 precision: str = "bf16", kv_precision: str | None = None, device: int = 0, max_batch: int = 1,
                 max_tokens: int = 0, tp_rank: int = 0, tp_size: int = 1, nccl_id: bytes | None = None,
                 synthetic_seed: int | None = None, synthetic_std: float = 0.02, eps: float = 1e-6):
        self.config = config
        self.stateDict = stateDict
        self.tokenizer = tokenizer
        self.position = np.zeros(1, np.int32)
        ncfg = native_config(config, precision, kv_precision, max_batch, max_tokens, eps=eps)
        self.native = native.NativeModel(ncfg, device, tp_rank, tp_size, nccl_id)
        if stateDict is not None and stateDict.weightsDirectory is not None:
            self.native.load_state_dict_pb(stateDict.weightsDirectory)
        elif stateDict is not None:
            for k, v in stateDict.items():
                self.native.load_tensor(k, v)
        elif synthetic_seed is not None:
            self.native.init_synthetic(synthetic_seed, synthetic_std)
        else:
            raise ValueError("either a StateDictionary or synthetic_seed is required")
        self.native.finalize()
        self.compiledModel = CompiledModel(self)
        self.model = AutoregressiveModel(self)

    def getConfig(self):
        return self.config

    def getCompiledModel(self) -> CompiledModel:
        return self.compiledModel

    def getAutoregressiveModel(self) -> AutoregressiveModel:
        return self.model

    def getPosition(self) -> np.ndarray:
        return self.position

    def getTokenizer(self):
        return self.tokenizer

    def getTokenEmbeddings(self):
        return None if self.stateDict is None else self.stateDict.get("model.embed_tokens.weight")

    def setTemperature(self, t: float, seed: int | None = None):
        """Qwen3.setTemperature (Qwen3.java:285-291): 0 for greedy decoding."""
        self.model.setTemperature(t, seed)

    def generate(self, prompt_tokens, steps: int) -> np.ndarray:
        """Generation of `steps` tokens (prompt included) entirely on the device, greedy or sampled per
        setTemperature."""
        return self.native.generate(np.asarray(prompt_tokens, np.int32), steps)

    def close(self):
        self.native.close()
