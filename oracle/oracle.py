"""ctypes wrapper of the CPU oracle (oracle/qwen3_oracle.c) -- TEST INFRASTRUCTURE ONLY.

The oracle restates the reference's Qwen3 forward step on the CPU (fp64 or fp32) and is
the parity checker for the CUDA library.  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline / reference legs use it; the product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")


class OrefConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("dim", "hidden_dim", "layers", "heads", "kv_heads", "head_dim", "vocab",
                                       "seq_len", "shared_weights", "qk_norm_mode", "has_qkv_bias", "share_layers")] + \
               [("rope_theta", C.c_double), ("eps", C.c_double)]


def build() -> None:
    """Compile both precisions with the committed Makefile (no-op when up to date)."""
    r = subprocess.run(["make", "-s", "-C", HERE], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + r.stdout + r.stderr)


_libs: dict[str, C.CDLL] = {}


def lib(precision: str = "f64") -> C.CDLL:
    if precision not in ("f64", "f32"):
        raise ValueError(precision)
    if precision not in _libs:
        path = os.path.join(BUILD, f"liboracle_{precision}.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        s = "_" + precision
        P, D, I, F = C.c_void_p, C.POINTER(C.c_double), C.c_int, C.POINTER(C.c_float)
        sig = {
            "oref_create": (P, [C.POINTER(OrefConfig)]),
            "oref_destroy": (None, [P]),
            "oref_set": (I, [P, C.c_char_p, F, C.c_longlong]),
            "oref_reset": (None, [P]),
            "oref_forward_token": (I, [P, I, I, F]),
            "oref_forward_hidden": (I, [P, F, I, F]),
            "oref_generate": (I, [P, C.POINTER(C.c_int), I, I, C.POINTER(C.c_int), F]),
            "oref_init_synthetic": (None, [P, C.c_uint64, C.c_float]),
            "oref_round_weights_bf16": (None, [P]),
            "oref_synth_value": (C.c_float, [C.c_uint64, C.c_uint32, C.c_uint64, C.c_float]),
            "oref_rope_freqs": (None, [C.c_double, I, I, D]),
            "oref_gqa_expand": (None, [D, I, I, I, D]),
            "oref_attention_keys": (None, [D, D, I, I, I, D]),
            "oref_attention_values": (None, [D, D, I, I, I, D]),
            "oref_causal_mask": (None, [D, I, I, I]),
            "oref_softmax": (None, [D, I, I]),
            "oref_rmsnorm": (None, [D, D, I, C.c_double, D]),
            "oref_argmax": (I, [F, I]),
            "oref_num_threads": (I, []),
            "oref_set_threads": (None, [I]),
            "oref_bench_slice": (I, [P, I, I, I, I]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name + s)
            fn.restype = res
            fn.argtypes = args
            setattr(L, name, fn)
        _libs[precision] = L
    return _libs[precision]


def _dp(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_double))


def _fp(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


# ------------------------------------------------------------------ component functions (KATs)
def rope_freqs(theta: float, head_dim: int, seq_len: int, precision="f64") -> np.ndarray:
    out = np.zeros((seq_len, head_dim // 2, 2), np.float64)
    lib(precision).oref_rope_freqs(theta, head_dim, seq_len, _dp(out))
    return out


def gqa_expand(x: np.ndarray, kv_heads: int, heads: int, head_dim: int, precision="f64") -> np.ndarray:
    x = np.ascontiguousarray(x, np.float64)
    out = np.zeros(heads * head_dim, np.float64)
    lib(precision).oref_gqa_expand(_dp(x), kv_heads, heads, head_dim, _dp(out))
    return out


def attention_keys(q: np.ndarray, K: np.ndarray, precision="f64") -> np.ndarray:
    heads, d = q.shape
    S = K.shape[0]
    q = np.ascontiguousarray(q, np.float64)
    K = np.ascontiguousarray(K, np.float64)
    out = np.zeros((heads, S), np.float64)
    lib(precision).oref_attention_keys(_dp(q), _dp(K), heads, d, S, _dp(out))
    return out


def attention_values(a: np.ndarray, V: np.ndarray, precision="f64") -> np.ndarray:
    heads, S = a.shape
    d = V.shape[2]
    a = np.ascontiguousarray(a, np.float64)
    V = np.ascontiguousarray(V, np.float64)
    out = np.zeros((heads, d), np.float64)
    lib(precision).oref_attention_values(_dp(a), _dp(V), heads, d, S, _dp(out))
    return out


def causal_mask(s: np.ndarray, pos: int, precision="f64") -> np.ndarray:
    s = np.array(s, np.float64, copy=True, order="C")
    lib(precision).oref_causal_mask(_dp(s), s.shape[0], s.shape[1], pos)
    return s


def softmax(x: np.ndarray, precision="f64") -> np.ndarray:
    x = np.array(x, np.float64, copy=True, order="C")
    lib(precision).oref_softmax(_dp(x), x.shape[0], x.shape[1])
    return x


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float, precision="f64") -> np.ndarray:
    x = np.ascontiguousarray(x, np.float64)
    w = np.ascontiguousarray(w, np.float64)
    out = np.zeros_like(x)
    lib(precision).oref_rmsnorm(_dp(x), _dp(w), x.size, eps, _dp(out))
    return out


def argmax(v: np.ndarray) -> int:
    v = np.ascontiguousarray(v, np.float32)
    return int(lib("f64").oref_argmax(_fp(v), v.size))


def synth_value(seed: int, tensor_id: int, idx: int, scale: float) -> float:
    return float(lib("f64").oref_synth_value(seed, tensor_id, idx, scale))


def num_threads(precision: str = "f64") -> int:
    return int(lib(precision).oref_num_threads())


def set_threads(n: int) -> None:
    """OpenMP threads of both oracle builds (overrides OMP_NUM_THREADS, which torchrun sets to 1)."""
    for p in ("f64", "f32"):
        lib(p).oref_set_threads(int(n))


# ------------------------------------------------------------------ full model
class OracleModel:
    """The reference's Qwen3 (Appendix semantics in qwen3_oracle.c) on the CPU.

    cfg keys: dim, hidden_dim, layers, heads, kv_heads, head_dim, vocab, seq_len,
    shared_weights, qk_norm (0/1/2), has_qkv_bias, rope_theta, eps.
    """

    def __init__(self, cfg: dict, precision: str = "f64"):
        self.cfg = dict(cfg)
        self.L = lib(precision)
        c = OrefConfig(cfg["dim"], cfg["hidden_dim"], cfg["layers"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"],
                       cfg["vocab"], cfg["seq_len"], int(cfg.get("shared_weights", 0)), int(cfg.get("qk_norm", 1)),
                       int(cfg.get("has_qkv_bias", 0)), int(cfg.get("share_layers", 0)), float(cfg.get("rope_theta", 1e6)), float(cfg.get("eps", 1e-6)))
        self._h = self.L.oref_create(C.byref(c))
        if not self._h:
            raise MemoryError("oracle allocation failed")

    def close(self):
        if self._h:
            self.L.oref_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set(self, key: str, arr) -> None:
        a = np.ascontiguousarray(np.asarray(arr, dtype=np.float32))
        r = self.L.oref_set(self._h, key.encode(), _fp(a), a.size)
        if r == -1:
            return  # key not used by this configuration (e.g. lm_head when tied)
        if r != 0:
            raise ValueError(f"oracle: bad tensor {key} ({a.shape})")

    def load_state_dict(self, sd: dict) -> None:
        for k, v in sd.items():
            self.set(k, v)

    def init_synthetic(self, seed: int, std: float) -> None:
        self.L.oref_init_synthetic(self._h, seed, std)

    def round_weights_bf16(self) -> None:
        self.L.oref_round_weights_bf16(self._h)

    def reset(self) -> None:
        self.L.oref_reset(self._h)

    def forward_token(self, token: int, pos: int) -> np.ndarray:
        out = np.zeros(self.cfg["vocab"], np.float32)
        if self.L.oref_forward_token(self._h, int(token), int(pos), _fp(out)):
            raise ValueError("oracle: token/position out of range")
        return out

    def forward_hidden(self, x: np.ndarray, pos: int) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(self.cfg["vocab"], np.float32)
        if self.L.oref_forward_hidden(self._h, _fp(x), int(pos), _fp(out)):
            raise ValueError("oracle: position out of range")
        return out

    def bench_slice(self, layer: int, pos: int, lm_r0: int, lm_r1: int) -> None:
        if self.L.oref_bench_slice(self._h, layer, pos, lm_r0, lm_r1):
            raise ValueError("oracle: bad bench slice")

    def generate(self, prompt, steps: int):
        p = np.ascontiguousarray(prompt, np.int32)
        toks = np.zeros(steps, np.int32)
        last = np.zeros(self.cfg["vocab"], np.float32)
        r = self.L.oref_generate(self._h, p.ctypes.data_as(C.POINTER(C.c_int)), p.size, steps,
                                 toks.ctypes.data_as(C.POINTER(C.c_int)), _fp(last))
        if r:
            raise ValueError("oracle: generate failed")
        return toks, last


# ------------------------------------------------------------------ sampling (test infrastructure)
class JavaRandom:
    """java.util.Random restated (the published 48-bit linear congruential generator), so that tests can
    reproduce the draws of a Java caller seeding new Random(seed)."""

    MASK = (1 << 48) - 1

    def __init__(self, seed: int):
        self.s = (seed ^ 0x5DEECE66D) & self.MASK

    def next(self, bits: int) -> int:
        self.s = (self.s * 0x5DEECE66D + 0xB) & self.MASK
        v = self.s >> (48 - bits)
        return v - (1 << 32) if v >= (1 << 31) else v  # Java's (int) cast

    def next_double(self) -> float:
        return ((self.next(26) << 27) + self.next(27)) * 2.0 ** -53


def sample_token(values, vocab: int, temperature: float, top_p: float, r: float | None) -> int:
    """AutoregressiveModel.sampleToken (engine/ml/src/main/java/org/almostrealism/ml/AutoregressiveModel.java:323-386)
    in double precision, with the uniform draw r given (None or temperature <= 0: greedy first max)."""
    v = np.asarray(values, np.float64)[:vocab]
    if temperature <= 0.0 or r is None:
        return int(np.argmax(v))  # numpy's argmax keeps the first maximum, like the strict > loop
    probs = v / temperature
    probs = np.exp(probs - probs.max())
    probs = probs / probs.sum()
    if top_p < 1.0:
        order = np.argsort(-probs, kind="stable")  # Arrays.sort with a comparator is stable
        cum = np.cumsum(probs[order])
        cutoff = int(np.searchsorted(cum >= top_p, True)) + 1 if (cum >= top_p).any() else vocab
        top_sum = float(cum[cutoff - 1])
        keep = np.zeros(vocab, bool)
        keep[order[:cutoff]] = True
        probs = np.where(keep, probs, 0.0) / top_sum
    cumulative = np.cumsum(probs)
    idx = int(np.searchsorted(cumulative, r, side="right"))  # first i with r < cumulative[i]
    return min(idx, vocab - 1)


def sample_qwen3(logits, vocab: int, temperature: float, r: float | None) -> int:
    """The sampler Qwen3 generates with (AutoregressiveModel.of, AutoregressiveModel.java:405-434): logits divided by
    the temperature, softmax, then sampleToken(probabilities, vocab, 1.0, 1.0, random) -- a second softmax."""
    v = np.asarray(logits, np.float64)[:vocab]
    if temperature <= 0.0 or r is None:
        return int(np.argmax(v))
    p = v / temperature
    p = np.exp(p - p.max())
    p = p / p.sum()
    return sample_token(p, vocab, 1.0, 1.0, r)
