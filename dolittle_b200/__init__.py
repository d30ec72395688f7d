"""dolittle_b200: B200-native (sm_100a) Qwen3 token loop behind Dolittle's
CUDA-backend interfaces.

The compute path is the C ABI in include/dolittle_b200.h, implemented by
hand-written sm_100a kernels in dolittle_b200/csrc and built in-tree into
dolittle_b200/libdolittle_b200.so (`python -m dolittle_b200.build`).  There is
no CPU or library fallback: importing the engine without the library fails.
"""
from ._lib import (DL_BF16, DL_DECODE_KERNELS, DL_DECODE_PERSISTENT, DL_EVENT_CONSUMED, DL_EVENT_SELECTED,
                   DL_EVENT_TERMINAL, DL_F32, DL_PREFILL_FAST, DL_PREFILL_PARITY, DL_REASON_CANCELLED,
                   DL_REASON_EOS, DL_REASON_FAILURE, DL_REASON_LIMIT, DL_RNG_MT19937_64, DL_RNG_PHILOX4X32_10,
                   DolittleError, LIB_PATH, header_symbols, lib)
from .engine import QWEN3_8B, Engine, Generation, Qwen3Config, SelectionMode, Settings

__all__ = ["DL_BF16", "DL_DECODE_KERNELS", "DL_DECODE_PERSISTENT", "DL_EVENT_CONSUMED", "DL_EVENT_SELECTED",
           "DL_EVENT_TERMINAL", "DL_F32", "DL_PREFILL_FAST", "DL_PREFILL_PARITY", "DL_REASON_CANCELLED",
           "DL_REASON_EOS", "DL_REASON_FAILURE", "DL_REASON_LIMIT", "DL_RNG_MT19937_64", "DL_RNG_PHILOX4X32_10",
           "DolittleError", "LIB_PATH",
           "header_symbols", "lib", "QWEN3_8B", "Engine", "Generation", "Qwen3Config", "SelectionMode",
           "Settings"]
