"""ctypes binding of the C ABI in include/dolittle_b200.h.

The library is the in-tree build dolittle_b200/libdolittle_b200.so (sm_100a).
There is no fallback: when it is missing, loading raises ImportError.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdolittle_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "dolittle_b200.h")

DL_OK, DL_INVALID_ARGUMENT, DL_UNSUPPORTED, DL_CUDA_ERROR, DL_OUT_OF_MEMORY, DL_DEVICE_FAULT, DL_NOT_READY = range(7)
DL_EVENT_NONE, DL_EVENT_CONSUMED, DL_EVENT_SELECTED, DL_EVENT_TERMINAL = range(4)
DL_REASON_LIMIT, DL_REASON_EOS, DL_REASON_CANCELLED, DL_REASON_FAILURE = range(4)
DL_BF16, DL_F32 = 0, 1
DL_PREFILL_PARITY, DL_PREFILL_FAST = 0, 1
DL_DECODE_PERSISTENT, DL_DECODE_KERNELS = 0, 1
DL_RNG_MT19937_64, DL_RNG_PHILOX4X32_10 = 0, 1


class DolittleError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


class ModelConfig(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("query_heads", C.c_uint32), ("kv_heads", C.c_uint32),
                ("head_width", C.c_uint32), ("mlp_width", C.c_uint32), ("vocabulary", C.c_uint32),
                ("layers", C.c_uint32), ("epsilon", C.c_float), ("theta", C.c_double)]


class Sampling(C.Structure):
    _fields_ = [("mode", C.c_int32), ("temperature", C.c_double), ("top_k", C.c_size_t),
                ("top_p", C.c_double)]


class GenerationStats(C.Structure):
    _fields_ = [("prefill_ms", C.c_double), ("decode_ms", C.c_double), ("decode_steps", C.c_uint64),
                ("kernels_per_decode_step", C.c_uint64), ("kernels_total", C.c_uint64),
                ("status", C.c_uint32), ("fault", C.c_uint32)]


class SequenceEvent(C.Structure):
    _fields_ = [("kind", C.c_uint8), ("reason", C.c_uint8), ("reserved", C.c_uint16), ("status", C.c_uint32),
                ("position", C.c_uint64), ("count", C.c_uint64), ("token", C.c_uint32), ("norm", C.c_float)]


class ServeStats(C.Structure):
    _fields_ = [("prefill_ms", C.c_double), ("decode_ms", C.c_double), ("decode_steps", C.c_uint64),
                ("kernels_per_decode_step", C.c_uint64)]


_lib = None

vp, sz, u32p, u16p = C.c_void_p, C.c_size_t, C.POINTER(C.c_uint32), C.POINTER(C.c_uint16)
i64p = C.POINTER(C.c_int64)

SIGNATURES = {
    "dl_last_error": (C.c_char_p, []),
    "dl_version": (C.c_char_p, []),
    "dl_projection": (C.c_int, [C.c_int, vp, vp, vp, sz, sz, sz, vp, vp]),
    "dl_rms_norm": (C.c_int, [C.c_int, vp, vp, vp, sz, sz, C.c_float, vp]),
    "dl_rotary": (C.c_int, [C.c_int, vp, vp, sz, sz, sz, sz, C.c_double, vp, vp, C.c_int]),
    "dl_attention_scale": (C.c_int, [vp, sz, vp]),
    "dl_attention_workspace_bytes": (sz, [sz, sz, sz]),
    "dl_attention": (C.c_int, [C.c_int, vp, vp, vp, vp, sz, sz, sz, sz, vp, sz, vp, sz, vp, vp]),
    "dl_attention_prefill_fast_workspace_bytes": (sz, [sz, sz, sz]),
    "dl_attention_prefill_fast": (C.c_int, [vp, vp, vp, vp, sz, sz, sz, sz, vp, sz, sz, vp]),
    "dl_attention_fixed_scratch": (C.c_int, [C.c_int, vp, vp, vp, vp, sz, sz, sz, sz, vp, sz, vp, sz]),
    "dl_embedding": (C.c_int, [C.c_int, vp, vp, vp, sz, sz, vp]),
    "dl_add": (C.c_int, [C.c_int, vp, vp, vp, sz, vp]),
    "dl_silu_multiply": (C.c_int, [C.c_int, vp, vp, vp, sz, vp]),
    "dl_qkv_projection": (C.c_int, [vp, vp, C.c_float, vp, sz, sz, sz, sz, vp, vp, vp, vp, vp]),
    "dl_rope_inverse_frequency": (C.c_int, [vp, sz, C.c_double, vp]),
    "dl_qk_norm_rope_append": (C.c_int, [vp, vp, vp, vp, vp, vp, vp, vp, sz, sz, sz, sz, C.c_float, vp]),
    "dl_projection_residual": (C.c_int, [vp, vp, vp, sz, sz, sz, vp]),
    "dl_gemm_bf16": (C.c_int, [vp, sz, vp, vp, sz, sz, sz, sz, C.c_int, vp]),
    "dl_gemm_bf16_split_workspace_bytes": (sz, [sz, sz]),
    "dl_gemm_bf16_split": (C.c_int, [vp, sz, vp, vp, sz, sz, sz, sz, C.c_int, vp, vp, vp, sz]),
    "dl_gemm_bf16_config": (C.c_int, [vp, sz, vp, vp, sz, sz, sz, sz, C.c_int, vp, vp, vp, sz, C.c_int, C.c_int,
                                      C.c_int]),
    "dl_sampler_required_bytes": (sz, [sz]),
    "dl_sampler_create": (C.c_int, [sz, C.c_int, C.POINTER(vp)]),
    "dl_sampler_destroy": (None, [vp]),
    "dl_sampler_set_engine": (C.c_int, [vp, C.c_int]),
    "dl_sampler_start": (C.c_int, [vp, C.POINTER(Sampling), C.c_uint64, u32p, sz, vp]),
    "dl_sampler_submit": (C.c_int, [vp, vp, C.POINTER(Sampling), C.c_uint64, vp, C.POINTER(vp)]),
    "dl_sampler_submit_next": (C.c_int, [vp, vp, vp, C.POINTER(vp)]),
    "dl_intervene": (C.c_int, [vp, vp, vp, vp, sz, sz, sz, C.c_float, vp]),
    "dl_normalize_injection": (C.c_int, [vp, vp, vp, vp, sz, C.c_float, vp]),
    "dl_direction": (C.c_int, [C.c_int, vp, vp, sz, vp, vp, vp]),
    "dl_engine_tensor_count": (sz, [C.POINTER(ModelConfig)]),
    "dl_engine_tensor_shape": (C.c_int, [C.POINTER(ModelConfig), sz, C.POINTER(sz), C.POINTER(sz)]),
    "dl_engine_create": (C.c_int, [C.POINTER(ModelConfig), C.c_int, sz, sz, C.POINTER(vp)]),
    "dl_engine_destroy": (None, [vp]),
    "dl_engine_init_random": (C.c_int, [vp, C.c_uint64, C.c_float]),
    "dl_engine_set_tensor": (C.c_int, [vp, sz, vp, sz]),
    "dl_engine_get_tensor": (C.c_int, [vp, sz, vp, sz]),
    "dl_engine_tensor_device": (C.c_int, [vp, sz, C.POINTER(vp), C.POINTER(sz)]),
    "dl_engine_reset": (C.c_int, [vp]),
    "dl_engine_consume": (C.c_int, [vp, u32p, sz, C.c_int, u16p]),
    "dl_engine_position": (sz, [vp]),
    "dl_engine_set_capture": (C.c_int, [vp, C.c_int]),
    "dl_engine_read_capture": (C.c_int, [vp, sz, sz, u16p]),
    "dl_engine_set_observation": (C.c_int, [vp, vp, sz]),
    "dl_engine_set_intervention": (C.c_int, [vp, C.c_int, sz, C.c_float, C.POINTER(C.c_float)]),
    "dl_engine_set_decode_path": (C.c_int, [vp, C.c_int]),
    "dl_engine_set_sampler_engine": (C.c_int, [vp, C.c_int]),
    "dl_engine_set_injection": (C.c_int, [vp, C.c_int64, u16p, C.c_float]),
    "dl_engine_set_reconstruction_head": (C.c_int, [vp, u16p]),
    "dl_engine_reconstruct": (C.c_int, [vp, u32p, sz, u16p]),
    "dl_engine_read_kv": (C.c_int, [vp, sz, C.c_int, sz, sz, u16p]),
    "dl_engine_generate": (C.c_int, [vp, u32p, sz, sz, C.POINTER(Sampling), C.c_uint64, u32p, sz, C.c_int,
                                     u32p, C.POINTER(sz), u16p, C.POINTER(GenerationStats)]),
    "dl_engine_start": (C.c_int, [vp, u32p, sz, sz, C.POINTER(Sampling), C.c_uint64, u32p, sz, C.c_int]),
    "dl_engine_collect": (C.c_int, [vp, sz, C.c_int64, C.POINTER(SequenceEvent)]),
    "dl_engine_request_stop": (C.c_int, [vp]),
    "dl_engine_drain": (C.c_int, [vp, u32p, C.POINTER(sz), C.POINTER(GenerationStats)]),
    "dl_serve_create": (C.c_int, [C.POINTER(ModelConfig), C.c_int, sz, sz, sz, C.c_int, C.c_int, C.POINTER(vp)]),
    "dl_serve_destroy": (None, [vp]),
    "dl_serve_nccl_id": (C.c_int, [vp]),
    "dl_serve_connect": (C.c_int, [vp, vp]),
    "dl_serve_ipc_handle": (C.c_int, [vp, vp]),
    "dl_serve_connect_peers": (C.c_int, [vp, vp]),
    "dl_serve_init_random": (C.c_int, [vp, C.c_uint64, C.c_float]),
    "dl_serve_set_sampler_engine": (C.c_int, [vp, C.c_int]),
    "dl_serve_set_tensor": (C.c_int, [vp, sz, vp, sz]),
    "dl_serve_get_tensor": (C.c_int, [vp, sz, vp, sz]),
    "dl_serve_slice_shape": (C.c_int, [vp, sz, C.POINTER(sz), C.POINTER(sz), C.POINTER(sz), C.POINTER(sz)]),
    "dl_serve_prefill": (C.c_int, [vp, u32p, sz, C.POINTER(Sampling), C.c_uint64, u32p]),
    "dl_serve_decode": (C.c_int, [vp, sz, u32p, u16p, C.POINTER(ServeStats)]),
    "dl_serve_position": (sz, [vp]),
    "dl_serve_set_capture": (C.c_int, [vp, C.c_int]),
    "dl_serve_read_capture": (C.c_int, [vp, sz, sz, sz, u16p]),
    "dl_serve_set_steering": (C.c_int, [vp, C.c_int, sz, C.c_float, C.POINTER(C.c_float), C.POINTER(C.c_uint8),
                                        C.c_int64, sz]),
    "dl_serve_steering_strength": (C.c_int, [vp, C.POINTER(C.c_float)]),
    "dl_serve_set_step_fusion": (C.c_int, [vp, C.c_int]),
    "dl_gemm_bf16_parts_workspace_bytes": (sz, [sz, sz, sz, sz]),
    "dl_gemm_bf16_parts": (C.c_int, [vp, sz, vp, vp, sz, sz, sz, sz, C.c_int, sz, vp, vp]),
    "dl_attention_decode_batched_workspace_bytes": (sz, [sz, sz, sz, sz]),
    "dl_attention_decode_batched_plan": (C.c_int, [sz, sz, sz, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "dl_attention_decode_batched": (C.c_int, [vp, vp, sz, sz, sz, vp, sz, sz, sz, sz, vp, vp, vp]),
}


def header_symbols() -> list:
    """Every function the public header declares."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"DL_API\s+[\w\s\*]+?\b(dl_\w+)\s*\(", text)))


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m dolittle_b200.build` "
                              "(the sm_100a library is required; there is no CPU path)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != DL_OK:
        raise DolittleError(status, lib().dl_last_error().decode())
