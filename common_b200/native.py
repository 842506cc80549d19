"""ctypes binding of libqwen3_b200.so (the C ABI declared in include/qwen3_b200.h).

This is the same binding a Java host would write with Panama FFM or JNI: plain structs,
pointers and sizes.  The library must exist (built by ``common_b200.build``); there is no
fallback implementation.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("QW_LIB") or os.path.join(HERE, "lib", "libqwen3_b200.so")  # QW_LIB: another build

QW_OK = 0
STATUS_NAMES = {0: "QW_OK", 1: "QW_ERR_ARG", 2: "QW_ERR_SHAPE", 3: "QW_ERR_OOM", 4: "QW_ERR_CUDA", 5: "QW_ERR_NCCL",
                6: "QW_ERR_TIMEOUT", 7: "QW_ERR_STATE", 8: "QW_ERR_UNSUPPORTED", 9: "QW_ERR_KEY"}
DTYPE_F32, DTYPE_BF16, DTYPE_F64 = 0, 1, 2
QKNORM_NONE, QKNORM_VECTOR, QKNORM_HEAD = 0, 1, 2

# every symbol include/qwen3_b200.h declares
EXPORTS = ("qw_abi_version", "qw_build_info", "qw_get_unique_id", "qw_create", "qw_load_tensor", "qw_load_state_dict_pb",
           "qw_init_synthetic",
           "qw_finalize_weights", "qw_reset", "qw_reserve", "qw_decode_step", "qw_forward_hidden", "qw_prefill",
           "qw_generate", "qw_decode_step_device", "qw_capture_decode", "qw_replay_decode", "qw_synchronize",
           "qw_stream", "qw_last_launch_count", "qw_last_error", "qw_destroy", "qw_profile_decode",
           "qw_set_device_inputs", "qw_profile_prefill", "qw_op_lm_head_argmax", "qw_op_lm_head_argmax_static", "qw_op_linear", "qw_set_sampling", "qw_decode_sample", "qw_op_sample")
KERNEL_NAMES = {0: "other", 1: "qkv", 2: "attn", 3: "o_proj", 4: "gate_up", 5: "down", 6: "lm_head", 7: "step"}


class QwConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "dim", "hidden_dim", "layers", "heads", "kv_heads", "head_dim", "vocab", "seq_len", "shared_weights",
        "qk_norm", "has_qkv_bias", "weight_dtype", "kv_dtype", "max_batch", "max_tokens", "page_size", "num_pages",
        "decode_kernels", "wait_limit_us", "test_stall_cta")] + \
        [("reserved", C.c_int32 * 2), ("rope_theta", C.c_double), ("eps", C.c_double)]


class QwenError(RuntimeError):
    """A non-zero qw_status (the Java shim raises HardwareException for the same)."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


_lib = None


def load() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m common_b200.build` "
                           "(the CUDA library is required; there is no CPU fallback)")
    L = C.CDLL(LIB_PATH)
    P, I32, PI = C.c_void_p, C.c_int32, C.POINTER(C.c_int32)
    PF = C.POINTER(C.c_float)
    sig = {
        "qw_abi_version": (I32, []),
        "qw_build_info": (C.c_char_p, []),
        "qw_get_unique_id": (I32, [P]),
        "qw_create": (I32, [C.POINTER(QwConfig), I32, I32, I32, P, C.POINTER(P)]),
        "qw_load_tensor": (I32, [P, C.c_char_p, I32, C.POINTER(C.c_int64), I32, P]),
        "qw_load_state_dict_pb": (I32, [P, C.c_char_p, C.POINTER(I32)]),
        "qw_init_synthetic": (I32, [P, C.c_uint64, C.c_float]),
        "qw_finalize_weights": (I32, [P]),
        "qw_reset": (I32, [P, I32]),
        "qw_reserve": (I32, [P, I32, I32]),
        "qw_decode_step": (I32, [P, PI, PI, PI, I32, PF, PI]),
        "qw_forward_hidden": (I32, [P, PF, PI, PI, I32, PF, PI]),
        "qw_prefill": (I32, [P, PI, PI, I32, I32, PF, PI]),
        "qw_generate": (I32, [P, PI, I32, I32, I32, PI]),
        "qw_decode_step_device": (I32, [P, P, P, P, I32, P, P, I32]),
        "qw_capture_decode": (I32, [P, P, P, P, I32, P, P]),
        "qw_replay_decode": (I32, [P, I32]),
        "qw_synchronize": (I32, [P]),
        "qw_profile_prefill": (I32, [P, PI, PI, I32, I32, PF, PI, I32, PI]),
        "qw_stream": (P, [P]),
        "qw_last_launch_count": (I32, [P]),
        "qw_last_error": (C.c_char_p, [P]),
        "qw_destroy": (None, [P]),
        "qw_profile_decode": (I32, [P, I32, PF, PI, I32, PI]),
        "qw_set_device_inputs": (I32, [P, PI, PI, I32]),
        "qw_op_lm_head_argmax": (I32, [P, I32, I32, I32, P, P, C.c_double, I32, P, P, P]),
        "qw_set_sampling": (I32, [P, C.c_double, C.c_double, C.c_int64, I32]),
        "qw_decode_sample": (I32, [P, PI, PI, PI, I32, PI]),
        "qw_op_sample": (I32, [P, I32, I32, I32, C.c_double, C.c_double, I32, P, P, P, P]),
        "qw_op_linear": (I32, [P, I32, I32, P, I32, I32, P, P, P, P]),
        "qw_op_lm_head_argmax_static": (I32, [P, I32, I32, I32, P, P, C.c_double, I32, P, P, P]),
    }
    for name, (res, args) in sig.items():
        if os.environ.get("QW_LIB") and not hasattr(L, name):
            continue  # another build (QW_LIB) may predate an entry point
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _ip(a):
    return None if a is None else a.ctypes.data_as(C.POINTER(C.c_int32))


def _fp(a):
    return None if a is None else a.ctypes.data_as(C.POINTER(C.c_float))


def make_config(dim, hidden_dim, layers, heads, kv_heads, head_dim, vocab, seq_len, shared_weights=False,
                qk_norm=QKNORM_VECTOR, has_qkv_bias=False, weight_dtype=DTYPE_BF16, kv_dtype=DTYPE_BF16,
                max_batch=1, max_tokens=0, page_size=64, num_pages=0, rope_theta=1e6, eps=1e-6,
                decode_kernels=0, wait_limit_us=0, test_stall_cta=0) -> QwConfig:
    c = QwConfig()
    c.dim, c.hidden_dim, c.layers, c.heads, c.kv_heads, c.head_dim = dim, hidden_dim, layers, heads, kv_heads, head_dim
    c.vocab, c.seq_len, c.shared_weights, c.qk_norm, c.has_qkv_bias = vocab, seq_len, int(shared_weights), qk_norm, int(has_qkv_bias)
    c.weight_dtype, c.kv_dtype, c.max_batch, c.max_tokens = weight_dtype, kv_dtype, max_batch, max_tokens or max_batch
    c.page_size, c.num_pages, c.rope_theta, c.eps = page_size, num_pages, rope_theta, eps
    c.decode_kernels = decode_kernels
    c.wait_limit_us, c.test_stall_cta = wait_limit_us, test_stall_cta
    return c


def op_error() -> str:
    return load().qw_last_error(None).decode()


def op_lm_head_argmax(w_ptr: int, w_dtype: int, vocab: int, dim: int, x_ptr: int, norm_ptr: int, eps: float,
                      batch: int, logits_ptr: int, argmax_ptr: int, stream: int = 0) -> None:
    """qw_op_lm_head_argmax over raw device pointers."""
    st = load().qw_op_lm_head_argmax(w_ptr, w_dtype, vocab, dim, x_ptr, norm_ptr, eps, batch, logits_ptr or None,
                                     argmax_ptr, stream or None)
    if st:
        raise QwenError(st, op_error())


def op_sample(logits_ptr: int, rows: int, vocab: int, ld: int, temperature: float, top_p: float, mode: int,
              r_ptr: int, scratch_ptr: int, out_ptr: int, stream: int = 0) -> None:
    """qw_op_sample over raw device pointers."""
    st = load().qw_op_sample(logits_ptr, rows, vocab, ld, temperature, top_p, mode, r_ptr or None,
                             scratch_ptr or None, out_ptr, stream or None)
    if st:
        raise QwenError(st, op_error())


LINEAR_STORE, LINEAR_RESID, LINEAR_SWIGLU = 0, 1, 2


def op_linear(w_ptr: int, n_out: int, k: int, x_ptr: int, t: int, epi: int, bias_ptr: int, resid_ptr: int,
              out_ptr: int, stream: int = 0) -> None:
    """qw_op_linear (tcgen05 GEMM) over raw device pointers."""
    st = load().qw_op_linear(w_ptr, n_out, k, x_ptr, t, epi, bias_ptr or None, resid_ptr or None, out_ptr,
                             stream or None)
    if st:
        raise QwenError(st, op_error())


def op_lm_head_argmax_static(w_ptr: int, w_dtype: int, vocab: int, dim: int, x_ptr: int, norm_ptr: int,
                             eps: float, batch: int, logits_ptr: int, argmax_ptr: int, stream: int = 0) -> None:
    """qw_op_lm_head_argmax_static over raw device pointers (scratch in the library's static array)."""
    st = load().qw_op_lm_head_argmax_static(w_ptr, w_dtype, vocab, dim, x_ptr, norm_ptr, eps, batch,
                                            logits_ptr or None, argmax_ptr, stream or None)
    if st:
        raise QwenError(st, op_error())


def unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    st = load().qw_get_unique_id(buf)
    if st:
        raise QwenError(st, "ncclGetUniqueId failed")
    return buf.raw


class NativeModel:
    """Owns one qw_model handle (one GPU, one tensor-parallel rank)."""

    def __init__(self, cfg: QwConfig, device: int = 0, tp_rank: int = 0, tp_size: int = 1, nccl_id: bytes | None = None):
        self.L = load()
        self.cfg = cfg
        h = C.c_void_p()
        idbuf = C.create_string_buffer(nccl_id, 128) if nccl_id else None
        st = self.L.qw_create(C.byref(cfg), device, tp_rank, tp_size, idbuf, C.byref(h))
        if st:
            raise QwenError(st, "qw_create failed (see stderr)")
        self.h = h

    def _check(self, st):
        if st:
            raise QwenError(st, self.L.qw_last_error(self.h).decode())

    def close(self):
        if getattr(self, "h", None):
            self.L.qw_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_tensor(self, key: str, arr: np.ndarray):
        a = np.ascontiguousarray(arr)
        if a.dtype == np.float32:
            dt = DTYPE_F32
        elif a.dtype == np.float64:
            dt = DTYPE_F64
        elif a.dtype == np.uint16:  # raw bf16 bits
            dt = DTYPE_BF16
        else:
            a = a.astype(np.float32)
            dt = DTYPE_F32
        dims = (C.c_int64 * a.ndim)(*a.shape)
        self._check(self.L.qw_load_tensor(self.h, key.encode(), dt, dims, a.ndim, a.ctypes.data_as(C.c_void_p)))

    def load_state_dict_pb(self, path: str) -> int:
        """Load a CollectionLibraryData file or directory; returns the number of tensors loaded."""
        n = C.c_int32(0)
        self._check(self.L.qw_load_state_dict_pb(self.h, os.fsencode(path), C.byref(n)))
        return n.value

    def init_synthetic(self, seed: int, std: float):
        self._check(self.L.qw_init_synthetic(self.h, seed, std))

    def finalize(self):
        self._check(self.L.qw_finalize_weights(self.h))

    def reset(self, slot: int = -1):
        self._check(self.L.qw_reset(self.h, slot))

    def reserve(self, slot: int, n_positions: int):
        self._check(self.L.qw_reserve(self.h, slot, n_positions))

    def decode_step(self, tokens, positions, slots=None, want_logits=True):
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        s = None if slots is None else np.ascontiguousarray(slots, np.int32)
        B = t.size
        logits = np.zeros((B, self.cfg.vocab), np.float32) if want_logits else None
        am = np.zeros(B, np.int32)
        self._check(self.L.qw_decode_step(self.h, _ip(t), _ip(s), _ip(p), B, _fp(logits), _ip(am)))
        return logits, am

    def forward_hidden(self, x, positions, slots=None, want_logits=True):
        x = np.ascontiguousarray(x, np.float32).reshape(-1, self.cfg.dim)
        p = np.ascontiguousarray(positions, np.int32)
        s = None if slots is None else np.ascontiguousarray(slots, np.int32)
        B = x.shape[0]
        logits = np.zeros((B, self.cfg.vocab), np.float32) if want_logits else None
        am = np.zeros(B, np.int32)
        self._check(self.L.qw_forward_hidden(self.h, _fp(x), _ip(s), _ip(p), B, _fp(logits), _ip(am)))
        return logits, am

    def prefill(self, tokens, slots=None, want_logits=True):
        t = np.ascontiguousarray(tokens, np.int32)
        if t.ndim == 1:
            t = t[None]
        B, S = t.shape
        s = None if slots is None else np.ascontiguousarray(slots, np.int32)
        logits = np.zeros((B, self.cfg.vocab), np.float32) if want_logits else None
        am = np.zeros(B, np.int32)
        self._check(self.L.qw_prefill(self.h, _ip(t), _ip(s), B, S, _fp(logits), _ip(am)))
        return logits, am

    def set_sampling(self, temperature: float, top_p: float = 1.0, seed: int = 0, mode: int = 0):
        self._check(self.L.qw_set_sampling(self.h, temperature, top_p, seed, mode))

    def decode_sample(self, tokens, positions, slots=None):
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        s = None if slots is None else np.ascontiguousarray(slots, np.int32)
        out = np.zeros(t.size, np.int32)
        self._check(self.L.qw_decode_sample(self.h, _ip(t), _ip(s), _ip(p), t.size, _ip(out)))
        return out

    def generate(self, prompts, steps: int):
        p = np.ascontiguousarray(prompts, np.int32)
        if p.ndim == 1:
            p = p[None]
        B, P = p.shape
        out = np.zeros((B, steps), np.int32)
        self._check(self.L.qw_generate(self.h, _ip(p), B, P, steps, _ip(out)))
        return out

    # device-pointer entry points (ints are raw CUDA device addresses)
    def decode_step_device(self, d_tokens, d_slots, d_positions, batch, d_logits, d_argmax, advance):
        self._check(self.L.qw_decode_step_device(self.h, d_tokens, d_slots, d_positions, batch, d_logits, d_argmax,
                                                 advance))

    def capture_decode(self, d_tokens, d_slots, d_positions, batch, d_logits, d_argmax):
        self._check(self.L.qw_capture_decode(self.h, d_tokens, d_slots, d_positions, batch, d_logits, d_argmax))

    def replay_decode(self, times: int):
        self._check(self.L.qw_replay_decode(self.h, times))

    def synchronize(self):
        self._check(self.L.qw_synchronize(self.h))

    def set_device_inputs(self, tokens, positions):
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        self._check(self.L.qw_set_device_inputs(self.h, _ip(t), _ip(p), t.size))

    def profile_decode(self, batch: int, cap: int = 4096):
        ms = np.zeros(cap, np.float32)
        kinds = np.zeros(cap, np.int32)
        n = C.c_int32(0)
        self._check(self.L.qw_profile_decode(self.h, batch, _fp(ms), _ip(kinds), cap, C.byref(n)))
        return ms[: n.value].copy(), kinds[: n.value].copy()

    def profile_prefill(self, tokens, slots=None, cap: int = 8192):
        """Per-kernel CUDA-event durations (ms) and classes of one prefill of (batch, seq_len) tokens."""
        t = np.ascontiguousarray(tokens, np.int32)
        s = None if slots is None else np.ascontiguousarray(slots, np.int32)
        ms = np.zeros(cap, np.float32)
        kinds = np.zeros(cap, np.int32)
        n = C.c_int32(0)
        self._check(self.L.qw_profile_prefill(self.h, _ip(t), _ip(s), t.shape[0], t.shape[1], _fp(ms), _ip(kinds), cap,
                                              C.byref(n)))
        return ms[: n.value].copy(), kinds[: n.value].copy()

    @property
    def stream(self) -> int:
        return self.L.qw_stream(self.h) or 0

    @property
    def last_launch_count(self) -> int:
        return self.L.qw_last_launch_count(self.h)
