"""ctypes view of the checker libraries.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs import this module.  It loads:

* ``liboracle.so`` -- the CPU restatement of the reference laws (dl_oracle.c);
* ``_ref/libref_host.so`` -- the reference's own BF16 and Categorical::select
  host code, compiled from the reference sources by oracle/Makefile;
* ``_ref/libref_cuda.so`` -- the reference's own CUDA kernels (compute_86 PTX,
  JIT-compiled by the driver on a B200) plus DeviceCategorical.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")


def reference_tree() -> str | None:
    """The reference source tree: $DOLITTLE_REFERENCE, else BASELINE.json's
    ``reference_path``; None when neither names an existing directory (the
    GPU box has no reference tree and uses the prebuilt _ref libraries)."""
    path = os.environ.get("DOLITTLE_REFERENCE")
    if not path:
        try:
            import json
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                path = json.load(f).get("reference_path")
        except (OSError, ValueError):
            path = None
    return path if path and os.path.isdir(os.path.join(path, "src")) else None


def build(reference: bool = True) -> None:
    """Compile the oracle (and, when the reference tree is present, _ref)."""
    targets = ["oracle"]
    ref = reference_tree() if reference else None
    if ref:
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE, *targets] + ([f"REF={ref}"] if ref else []), check=True)


class OrConfig(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("query_heads", C.c_uint32),
                ("kv_heads", C.c_uint32), ("head_width", C.c_uint32),
                ("mlp_width", C.c_uint32), ("vocabulary", C.c_uint32),
                ("layers", C.c_uint32), ("epsilon", C.c_float),
                ("theta", C.c_double)]


class OrIntervention(C.Structure):
    _fields_ = [("layer", C.c_int32), ("selected", C.c_uint64),
                ("strength", C.c_float), ("direction", C.POINTER(C.c_float)),
                ("state", C.POINTER(C.c_uint32))]


_lib = None


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build(reference=False)
        L = C.CDLL(path)
        sz = C.c_size_t
        L.or_bf16_from_float.restype = C.c_uint16
        L.or_bf16_from_float.argtypes = [C.c_float]
        L.or_bf16_to_float.restype = C.c_float
        L.or_bf16_to_float.argtypes = [C.c_uint16]
        L.or_bf16_from_float_array.argtypes = [f32p, u16p, sz]
        L.or_bf16_to_float_array.argtypes = [u16p, f32p, sz]
        L.or_projection.argtypes = [u16p, u16p, u16p, sz, sz, sz]
        L.or_projection_f32.argtypes = [u16p, u16p, f32p, sz, sz, sz]
        L.or_rms_norm.argtypes = [u16p, u16p, u16p, sz, sz, C.c_float]
        L.or_rope_inverse_frequency.restype = C.c_float
        L.or_rope_inverse_frequency.argtypes = [sz, sz, C.c_double]
        L.or_rotary.argtypes = [u16p, u16p, sz, sz, sz, sz, C.c_double]
        L.or_attention_scale.restype = C.c_float
        L.or_attention_scale.argtypes = [sz]
        L.or_attention.argtypes = [u16p, u16p, u16p, u16p, sz, sz, sz, sz, sz]
        L.or_add.argtypes = [u16p, u16p, u16p, sz]
        L.or_silu_multiply.argtypes = [u16p, u16p, u16p, sz]
        L.or_embedding.argtypes = [u32p, u16p, u16p, sz, sz]
        L.or_intervene.argtypes = [u16p, f32p, sz, sz, sz, sz, C.c_float, u32p]
        L.or_normalize_injection.restype = C.c_uint32
        L.or_normalize_injection.argtypes = [u16p, u16p, sz, C.c_float,
                                             C.POINTER(C.c_float)]
        L.or_steer_beta.restype = C.c_float
        L.or_steer_beta.argtypes = [u16p, sz, C.c_float]
        L.or_steer_rows.restype = C.c_uint32
        L.or_steer_rows.argtypes = [u16p, f32p, sz, sz, sz, sz, C.c_float]
        L.or_direction.restype = C.c_uint32
        L.or_direction.argtypes = [C.c_int, C.c_void_p, C.c_void_p, sz, f32p]
        L.or_mt64_seed.argtypes = [C.c_void_p, C.c_uint64]
        L.or_mt64_next.restype = C.c_uint64
        L.or_mt64_next.argtypes = [C.c_void_p]
        L.or_mt64_state_bytes.restype = sz
        L.or_select_host.restype = C.c_int
        L.or_select_host.argtypes = [f32p, sz, C.c_int, C.c_double, sz,
                                     C.c_double, C.c_uint64,
                                     C.POINTER(C.c_uint32)]
        L.or_select_device.argtypes = [f32p, sz, C.c_int, C.c_double, sz,
                                       C.c_double, C.c_uint64,
                                       C.POINTER(C.c_uint32),
                                       C.POINTER(C.c_uint32)]
        L.or_philox.argtypes = [C.c_uint64, C.c_uint32, C.c_uint64, u32p]
        L.or_fill_normal_bf16.argtypes = [u16p, sz, C.c_uint64, C.c_uint32,
                                          C.c_float]
        L.or_fill_uniform_ids.argtypes = [u32p, sz, C.c_uint64, C.c_uint32,
                                          C.c_uint32]
        L.or_forward.argtypes = [C.POINTER(OrConfig), C.POINTER(C.c_void_p),
                                 C.POINTER(C.c_void_p), sz, u32p, sz, sz,
                                 C.c_void_p, C.c_int32, C.c_void_p,
                                 C.POINTER(OrIntervention)]
        L.or_max_threads.restype = C.c_int
        L.or_set_threads.argtypes = [C.c_int]
        _lib = L
    return _lib


# --------------------------------------------------------------------------
# Array-level helpers
# --------------------------------------------------------------------------
def bf16_from_f32(a) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, np.uint16)
    lib().or_bf16_from_float_array(a.reshape(-1), out.reshape(-1), a.size)
    return out


def f32_from_bf16(a) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16)
    return (a.astype(np.uint32) << 16).view(np.float32)


def projection(x, w):
    x = np.ascontiguousarray(x, np.uint16)
    w = np.ascontiguousarray(w, np.uint16)
    rows, I = x.shape
    O = w.shape[0]
    y = np.empty((rows, O), np.uint16)
    lib().or_projection(x, w, y, rows, I, O)
    return y


def rms_norm(x, w, eps=1e-6):
    x = np.ascontiguousarray(x, np.uint16)
    rows, width = x.shape
    y = np.empty_like(x)
    lib().or_rms_norm(x, np.ascontiguousarray(w, np.uint16), y, rows, width, eps)
    return y


def rotary(x, first_position, theta):
    """x: [positions, heads, width] BF16 bits."""
    x = np.ascontiguousarray(x, np.uint16)
    p, h, w = x.shape
    y = np.empty_like(x)
    lib().or_rotary(x, y, p, h, w, first_position, theta)
    return y


def attention(q, k, v, first_position):
    """q: [rows, Hq, d]; k, v: [>= first+rows, Hkv, d] BF16 bits."""
    q = np.ascontiguousarray(q, np.uint16)
    k = np.ascontiguousarray(k, np.uint16)
    v = np.ascontiguousarray(v, np.uint16)
    rows, H, d = q.shape
    G = k.shape[1]
    y = np.empty_like(q)
    lib().or_attention(q, k, v, y, rows, H, G, d, first_position)
    return y


def add(a, b):
    a = np.ascontiguousarray(a, np.uint16)
    y = np.empty_like(a)
    lib().or_add(a, np.ascontiguousarray(b, np.uint16), y, a.size)
    return y


def silu_multiply(g, u):
    g = np.ascontiguousarray(g, np.uint16)
    y = np.empty_like(g)
    lib().or_silu_multiply(g, np.ascontiguousarray(u, np.uint16), y, g.size)
    return y


def fill_normal_bf16(n, seed, stream, scale):
    out = np.empty(n, np.uint16)
    lib().or_fill_normal_bf16(out, n, seed, stream, scale)
    return out


def uniform_ids(n, seed, stream, bound):
    out = np.empty(n, np.uint32)
    lib().or_fill_uniform_ids(out, n, seed, stream, bound)
    return out


def steer_beta(row_bits, alpha):
    """alpha * ||h|| with the one-row edit's norm law (FP32)."""
    r = np.ascontiguousarray(row_bits, np.uint16).reshape(-1)
    return np.float32(lib().or_steer_beta(r, r.size, alpha))


def steer_rows(rows_bits, direction, first_position, steer_from, beta):
    """Rows [n][D] at positions first_position + r: those >= steer_from get
    round(h + beta * u).  Returns (status, new rows)."""
    h = np.array(rows_bits, np.uint16, copy=True, order="C")
    u = np.ascontiguousarray(direction, np.float32)
    st = lib().or_steer_rows(h, u, h.shape[1], h.shape[0], first_position, steer_from, beta)
    return int(st), h


def direction(original, edited):
    """(status, FP32 direction) of the DeviceDirection law; inputs are BF16
    bits (uint16) or FP32 arrays of one width.  On status 1 the direction
    is all NaN (the law leaves its output untouched)."""
    bf16 = np.asarray(original).dtype == np.uint16
    dt = np.uint16 if bf16 else np.float32
    a = np.ascontiguousarray(original, dt).reshape(-1)
    b = np.ascontiguousarray(edited, dt).reshape(-1)
    out = np.full(a.size, np.nan, np.float32)
    status = lib().or_direction(int(bf16), a.ctypes.data, b.ctypes.data, a.size, out)
    return int(status), out


PHILOX_SAMPLER_STREAM = 0x5A4D504C


def philox_word(seed: int, k: int) -> int:
    """Draw k of the sampler's Philox4x32-10 stream under key `seed`: the
    first two words of the block at counter {k lo, k hi, 0x5A4D504C, 0}, low
    word first (the same generator as or_fill_normal_bf16)."""
    out = np.zeros(4, np.uint32)
    lib().or_philox(C.c_uint64(seed), PHILOX_SAMPLER_STREAM, C.c_uint64(k), out)
    return (int(out[1]) << 32) | int(out[0])


class MT64:
    """The std::mt19937_64 stream restated in dl_oracle.c."""

    def __init__(self, seed: int):
        self._buf = C.create_string_buffer(lib().or_mt64_state_bytes())
        lib().or_mt64_seed(self._buf, C.c_uint64(seed))

    def __call__(self) -> int:
        return lib().or_mt64_next(self._buf)


def select_host(logits, categorical, temperature=1.0, top_k=0, top_p=1.0,
                word=0):
    logits = np.ascontiguousarray(logits, np.float32)
    token = C.c_uint32(0)
    rc = lib().or_select_host(logits, logits.size, int(categorical),
                              temperature, top_k, top_p, C.c_uint64(word),
                              C.byref(token))
    return None if rc else token.value


def select_device(logits, categorical, temperature=1.0, top_k=0, top_p=1.0,
                  word=0):
    logits = np.ascontiguousarray(logits, np.float32)
    token, status = C.c_uint32(0), C.c_uint32(0)
    lib().or_select_device(logits, logits.size, int(categorical), temperature,
                           top_k, top_p, C.c_uint64(word), C.byref(token),
                           C.byref(status))
    return token.value, status.value


# --------------------------------------------------------------------------
# Model forward (reference recipe order) over host arrays
# --------------------------------------------------------------------------
ROLES = ("input_norm", "q", "k", "v", "q_norm", "k_norm", "o",
         "post_norm", "gate", "up", "down")


@dataclass
class Config:
    hidden: int
    query_heads: int
    kv_heads: int
    head_width: int
    mlp_width: int
    vocabulary: int
    layers: int
    epsilon: float = 1e-6
    theta: float = 1e6

    def c(self) -> OrConfig:
        return OrConfig(self.hidden, self.query_heads, self.kv_heads,
                        self.head_width, self.mlp_width, self.vocabulary,
                        self.layers, self.epsilon, self.theta)

    def shapes(self):
        D, Q = self.hidden, self.query_heads * self.head_width
        G, F = self.kv_heads * self.head_width, self.mlp_width
        d, V = self.head_width, self.vocabulary
        glob = [("embedding", (V, D)), ("final_norm", (D,)), ("lm_head", (V, D))]
        block = [("input_norm", (D,)), ("q", (Q, D)), ("k", (G, D)), ("v", (G, D)),
                 ("q_norm", (d,)), ("k_norm", (d,)), ("o", (D, Q)),
                 ("post_norm", (D,)), ("gate", (F, D)), ("up", (F, D)),
                 ("down", (D, F))]
        return glob, block


class OracleModel:
    """Weights (BF16 bits, host) + KV cache, stepping rows through or_forward."""

    def __init__(self, cfg: Config, tensors: list, capacity: int):
        self.cfg = cfg
        self.tensors = [np.ascontiguousarray(t, np.uint16) for t in tensors]
        self.capacity = capacity
        G = cfg.kv_heads * cfg.head_width
        self.cache = [np.zeros((capacity, G), np.uint16)
                      for _ in range(2 * cfg.layers)]
        self._tp = (C.c_void_p * len(self.tensors))(
            *[t.ctypes.data for t in self.tensors])
        self._cp = (C.c_void_p * len(self.cache))(
            *[c.ctypes.data for c in self.cache])

    def forward(self, tokens, first_position, logits=True, capture_layer=-1,
                edit=None):
        tokens = np.ascontiguousarray(tokens, np.uint32)
        rows = tokens.size
        out = np.empty(self.cfg.vocabulary, np.uint16) if logits else None
        if capture_layer == -2:      # every block output, [layers][rows][D]
            cap = np.empty((self.cfg.layers, rows, self.cfg.hidden), np.uint16)
        elif capture_layer >= 0:
            cap = np.empty((rows, self.cfg.hidden), np.uint16)
        else:
            cap = None
        cfg = self.cfg.c()
        lib().or_forward(C.byref(cfg), self._tp, self._cp, self.capacity,
                         tokens, rows, first_position,
                         out.ctypes.data if out is not None else None,
                         capture_layer,
                         cap.ctypes.data if cap is not None else None,
                         C.byref(edit) if edit is not None else None)
        return out, cap


def tensor_list(cfg: Config, named: dict) -> list:
    glob, block = cfg.shapes()
    out = [named[n] for n, _ in glob]
    for layer in range(cfg.layers):
        out += [named[f"layers.{layer}.{n}"] for n, _ in block]
    return out


# --------------------------------------------------------------------------
# Reference libraries compiled from the reference sources (oracle/_ref)
# --------------------------------------------------------------------------
_ref_host = None
_ref_cuda = None


def ref_host():
    global _ref_host
    if _ref_host is None:
        path = os.path.join(REF_DIR, "libref_host.so")
        if not os.path.exists(path):
            return None
        L = C.CDLL(path)
        L.ref_bf16_from_float.restype = C.c_uint16
        L.ref_bf16_from_float.argtypes = [C.c_float]
        L.ref_bf16_to_float.restype = C.c_float
        L.ref_bf16_to_float.argtypes = [C.c_uint16]
        L.ref_rng_create.restype = C.c_void_p
        L.ref_rng_create.argtypes = [C.c_uint64]
        L.ref_rng_destroy.argtypes = [C.c_void_p]
        L.ref_rng_next.restype = C.c_uint64
        L.ref_rng_next.argtypes = [C.c_void_p]
        L.ref_rng_equal.restype = C.c_int
        L.ref_rng_equal.argtypes = [C.c_void_p, C.c_void_p]
        L.ref_categorical_select.restype = C.c_int
        L.ref_categorical_select.argtypes = [f32p, C.c_size_t, C.c_int,
                                             C.c_double, C.c_size_t,
                                             C.c_double, C.c_void_p,
                                             C.POINTER(C.c_uint32)]
        _ref_host = L
    return _ref_host


def ref_cuda():
    """The reference CUDA build, or None when it was not built."""
    global _ref_cuda
    if _ref_cuda is None:
        path = os.path.join(REF_DIR, "libref_cuda.so")
        if not os.path.exists(path):
            return None
        L = C.CDLL(path)
        sz, vp = C.c_size_t, C.c_void_p
        L.ref_projection.argtypes = [C.c_int, vp, vp, vp, sz, sz, sz, vp, vp]
        L.ref_rms_norm.argtypes = [C.c_int, vp, vp, vp, sz, sz, C.c_float, vp]
        L.ref_rotary.argtypes = [C.c_int, vp, vp, sz, sz, sz, sz, C.c_double,
                                 vp, vp, C.c_int]
        L.ref_attention_scale.argtypes = [vp, sz, vp]
        L.ref_attention.argtypes = [C.c_int, vp, vp, vp, vp, sz, sz, sz, sz,
                                    vp, sz, vp, sz, vp]
        L.ref_embedding.argtypes = [C.c_int, vp, vp, vp, sz, sz, vp]
        L.ref_add.argtypes = [C.c_int, vp, vp, vp, sz, vp]
        L.ref_silu_multiply.argtypes = [C.c_int, vp, vp, vp, sz, vp]
        L.ref_qwen3_scratch_bytes.restype = sz
        L.ref_qwen3_scratch_bytes.argtypes = [C.POINTER(OrConfig), sz]
        L.ref_qwen3_forward.argtypes = [C.POINTER(OrConfig),
                                        C.POINTER(C.c_void_p),
                                        C.POINTER(C.c_void_p), sz, vp, sz, sz,
                                        vp, C.c_int, vp, vp, vp]
        L.ref_device_select.argtypes = [f32p, sz, C.c_int, C.c_int, C.c_double,
                                        sz, C.c_double, C.c_uint64, u32p]
        L.ref_device_sequence.argtypes = [f32p, sz, C.c_int, C.c_double, sz,
                                          C.c_double, C.c_uint64, sz, u32p]
        L.ref_direction.argtypes = [C.c_int, C.c_void_p, C.c_void_p, sz, f32p,
                                    C.POINTER(C.c_uint32)]
        for name in ("ref_projection", "ref_rms_norm", "ref_rotary",
                     "ref_attention_scale", "ref_attention", "ref_embedding",
                     "ref_add", "ref_silu_multiply", "ref_qwen3_forward",
                     "ref_device_select", "ref_device_sequence", "ref_direction"):
            getattr(L, name).restype = C.c_int
        _ref_cuda = L
    return _ref_cuda


def ref_direction(original, edited):
    """(status, FP32 direction) from the reference's own DeviceDirection on
    the GPU (oracle/_ref/libref_cuda.so); direction all NaN on status 1."""
    L = ref_cuda()
    bf16 = np.asarray(original).dtype == np.uint16
    dt = np.uint16 if bf16 else np.float32
    a = np.ascontiguousarray(original, dt).reshape(-1)
    b = np.ascontiguousarray(edited, dt).reshape(-1)
    out = np.full(a.size, np.nan, np.float32)
    status = C.c_uint32(7)
    rc = L.ref_direction(int(bf16), a.ctypes.data, b.ctypes.data, a.size, out, C.byref(status))
    if rc:
        raise RuntimeError("reference DeviceDirection failed")
    return int(status.value), out
