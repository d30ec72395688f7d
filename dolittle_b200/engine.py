"""Host-side mirror of the reference's generation interface over the C ABI.

Names follow the reference: `Settings`/`SelectionMode` are
src/inference/sampling/sampler.h; `Engine.consume_view` is
CachedForwardPlan::consume_view (src/inference/executor.cpp:1397-1481);
`Engine.generate` is the live device loop of prepare_device_generation +
start_sequence + collect_sequence (src/inference/executor.cpp:1482-1716,
src/kernels/cuda/decode.cu:379-610) driven by generate()
(src/inference/generation.cpp:69-331).  Invalid settings raise ValueError
(the reference throws std::invalid_argument).
"""
from __future__ import annotations

import ctypes as C
import enum
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from ._lib import check, lib


class SelectionMode(enum.IntEnum):
    greedy = 0
    categorical = 1


@dataclass
class Settings:
    mode: SelectionMode = SelectionMode.greedy
    temperature: float = 1.0
    top_k: int = 0
    top_p: float = 1.0

    def c(self) -> _lib.Sampling:
        return _lib.Sampling(int(self.mode), float(self.temperature), int(self.top_k), float(self.top_p))


@dataclass
class Qwen3Config:
    hidden: int = 4096
    query_heads: int = 32
    kv_heads: int = 8
    head_width: int = 128
    mlp_width: int = 12288
    vocabulary: int = 151936
    layers: int = 36
    epsilon: float = 1e-6
    theta: float = 1e6

    def c(self) -> _lib.ModelConfig:
        return _lib.ModelConfig(self.hidden, self.query_heads, self.kv_heads, self.head_width,
                                self.mlp_width, self.vocabulary, self.layers, self.epsilon, self.theta)

    def tensor_count(self) -> int:
        return int(lib().dl_engine_tensor_count(C.byref(self.c())))

    def tensor_shape(self, index: int) -> tuple:
        r, c = C.c_size_t(), C.c_size_t()
        check(lib().dl_engine_tensor_shape(C.byref(self.c()), index, C.byref(r), C.byref(c)))
        return (r.value, c.value)


QWEN3_8B = Qwen3Config()


@dataclass
class Generation:
    tokens: list
    prefill_ms: float
    decode_ms: float
    decode_steps: int
    kernels_per_decode_step: int
    kernels_total: int
    status: int
    logits: np.ndarray | None = field(default=None, repr=False)


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint32)


class Engine:
    """Resident Qwen3 weights + KV cache + prefill/decode loop on one GPU."""

    def __init__(self, config: Qwen3Config, device: int = 0, capacity: int = 1024, max_rows: int = 8):
        self.config = config
        self.capacity = capacity
        h = C.c_void_p()
        check(lib().dl_engine_create(C.byref(config.c()), device, capacity, max_rows, C.byref(h)))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().dl_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- weights ---------------------------------------------------------
    def init_random(self, seed: int, sigma: float = 0.02) -> None:
        check(lib().dl_engine_init_random(self._h, seed, sigma))

    def set_tensor(self, index: int, bits: np.ndarray) -> None:
        b = np.ascontiguousarray(bits, dtype=np.uint16)
        check(lib().dl_engine_set_tensor(self._h, index, b.ctypes.data, b.nbytes))

    def get_tensor(self, index: int) -> np.ndarray:
        shape = self.config.tensor_shape(index)
        out = np.empty(shape, np.uint16)
        check(lib().dl_engine_get_tensor(self._h, index, out.ctypes.data, out.nbytes))
        return out

    def tensor_device(self, index: int) -> tuple:
        """(device address, row stride in elements) of a resident tensor."""
        p, s = C.c_void_p(), C.c_size_t()
        check(lib().dl_engine_tensor_device(self._h, index, C.byref(p), C.byref(s)))
        return int(p.value), int(s.value)

    def load_tensors(self, tensors: list) -> None:
        for i, t in enumerate(tensors):
            self.set_tensor(i, t)

    # ---- sequence ----------------------------------------------------------
    def reset(self) -> None:
        check(lib().dl_engine_reset(self._h))

    @property
    def position(self) -> int:
        return int(lib().dl_engine_position(self._h))

    def consume_view(self, tokens, mode: int = _lib.DL_PREFILL_PARITY) -> np.ndarray:
        """Consume tokens at the current position; BF16 logits of the last row."""
        t = _u32(tokens)
        out = np.empty(self.config.vocabulary, np.uint16)
        check(lib().dl_engine_consume(self._h, t.ctypes.data_as(_lib.u32p), t.size, mode,
                                      out.ctypes.data_as(_lib.u16p)))
        return out

    def set_capture(self, layer: int) -> None:
        check(lib().dl_engine_set_capture(self._h, layer))

    def read_capture(self, first: int, count: int) -> np.ndarray:
        out = np.empty((count, self.config.hidden), np.uint16)
        check(lib().dl_engine_read_capture(self._h, first, count, out.ctypes.data_as(_lib.u16p)))
        return out

    def set_observation(self, device_rows_ptr: int | None, positions: int = 0) -> None:
        """Every block's output rows of later prompt passes go to the caller's
        device buffer [layers][positions][hidden] (BF16); None turns it off."""
        check(lib().dl_engine_set_observation(self._h, device_rows_ptr or None,
                                              positions if device_rows_ptr else 0))

    def set_intervention(self, layer: int, selected: int = 0, strength: float = 0.0, direction=None) -> None:
        d = np.ascontiguousarray(direction if direction is not None else np.zeros(self.config.hidden),
                                 dtype=np.float32)
        check(lib().dl_engine_set_intervention(self._h, layer, selected, strength,
                                               d.ctypes.data_as(C.POINTER(C.c_float))))

    def set_decode_path(self, path: int) -> None:
        """DL_DECODE_PERSISTENT (one cooperative kernel per token) or
        DL_DECODE_KERNELS (per-operation kernels); the results are identical."""
        check(lib().dl_engine_set_decode_path(self._h, path))

    def set_sampler_engine(self, engine: int) -> None:
        """Draw source of later categorical generations: DL_RNG_MT19937_64
        (the reference's stream, default) or DL_RNG_PHILOX4X32_10."""
        check(lib().dl_engine_set_sampler_engine(self._h, engine))

    def set_injection(self, position: int, source_bits=None, scale: float = 150.0) -> None:
        """Verbalizer injection: prompt position `position` gets
        BF16((h/||h||) * scale) of the BF16 row `source_bits` instead of its
        embedding; position < 0 clears it (ValueError on a zero/non-finite h)."""
        if position < 0:
            check(lib().dl_engine_set_injection(self._h, -1, None, 0.0))
            return
        h = np.ascontiguousarray(source_bits, np.uint16)
        if h.size != self.config.hidden:
            raise ValueError("injection source must have the hidden width")
        check(lib().dl_engine_set_injection(self._h, position, h.ctypes.data_as(_lib.u16p), scale))

    def set_reconstruction_head(self, head_bits) -> None:
        w = np.ascontiguousarray(head_bits, np.uint16)
        if w.size != self.config.hidden ** 2:
            raise ValueError("reconstruction head must be D x D")
        check(lib().dl_engine_set_reconstruction_head(self._h, w.ctypes.data_as(_lib.u16p)))

    def reconstruct(self, tokens) -> np.ndarray:
        """AR forward-only: BF16 bits [D] of head(residual of the last token)."""
        t = _u32(tokens)
        out = np.empty(self.config.hidden, np.uint16)
        check(lib().dl_engine_reconstruct(self._h, t.ctypes.data_as(_lib.u32p), t.size, out.ctypes.data_as(_lib.u16p)))
        return out

    def read_kv(self, layer: int, values: bool, first: int, count: int) -> np.ndarray:
        g = self.config.kv_heads * self.config.head_width
        out = np.empty((count, g), np.uint16)
        check(lib().dl_engine_read_kv(self._h, layer, int(values), first, count, out.ctypes.data_as(_lib.u16p)))
        return out

    # ---- device-side sequence loop (DeviceSequence) ---------------------
    def start(self, prompt, max_new: int, settings: Settings | None = None, seed: int = 0, stop_ids=(),
              prefill: int = _lib.DL_PREFILL_PARITY) -> None:
        """Enqueue the prompt pass, the first selection and the device loop
        of up to max_new selections; returns at once (see collect/drain)."""
        settings = settings or Settings()
        p = _u32(prompt)
        stops = _u32(list(stop_ids) or [0])
        s = settings.c()
        check(lib().dl_engine_start(self._h, p.ctypes.data_as(_lib.u32p), p.size, max_new, C.byref(s), seed,
                                    stops.ctypes.data_as(_lib.u32p), len(stop_ids), prefill))
        self._max_new = max_new  # the running sequence's budget (drain's buffer size)

    def collect(self, index: int, timeout_ms: int = -1):
        """Journal event `index` (0: prompt consumed, k: k-th selection, then
        a terminal event), or None if it did not arrive in time."""
        ev = _lib.SequenceEvent()
        st = lib().dl_engine_collect(self._h, index, timeout_ms, C.byref(ev))
        if st == _lib.DL_NOT_READY:
            return None
        check(st)
        return ev

    def request_stop(self) -> None:
        check(lib().dl_engine_request_stop(self._h))

    def drain(self) -> Generation:
        out = np.zeros(max(1, getattr(self, "_max_new", 0)), np.uint32)
        n = C.c_size_t()
        stats = _lib.GenerationStats()
        check(lib().dl_engine_drain(self._h, out.ctypes.data_as(_lib.u32p), C.byref(n), C.byref(stats)))
        return Generation(tokens=out[:n.value].tolist(), prefill_ms=stats.prefill_ms, decode_ms=stats.decode_ms,
                          decode_steps=int(stats.decode_steps),
                          kernels_per_decode_step=int(stats.kernels_per_decode_step),
                          kernels_total=int(stats.kernels_total), status=int(stats.status))

    def generate(self, prompt, max_new: int, settings: Settings | None = None, seed: int = 0,
                 stop_ids=(), prefill: int = _lib.DL_PREFILL_PARITY, want_logits: bool = False) -> Generation:
        settings = settings or Settings()
        p = _u32(prompt)
        stops = _u32(list(stop_ids) or [0])
        out = np.zeros(max_new, np.uint32)
        n_out = C.c_size_t()
        logits = np.empty((max_new, self.config.vocabulary), np.uint16) if want_logits else None
        stats = _lib.GenerationStats()
        s = settings.c()
        check(lib().dl_engine_generate(
            self._h, p.ctypes.data_as(_lib.u32p), p.size, max_new, C.byref(s), seed,
            stops.ctypes.data_as(_lib.u32p), len(stop_ids), prefill, out.ctypes.data_as(_lib.u32p),
            C.byref(n_out), logits.ctypes.data_as(_lib.u16p) if logits is not None else None,
            C.byref(stats)))
        n = n_out.value
        return Generation(tokens=out[:n].tolist(), prefill_ms=stats.prefill_ms, decode_ms=stats.decode_ms,
                          decode_steps=int(stats.decode_steps),
                          kernels_per_decode_step=int(stats.kernels_per_decode_step),
                          kernels_total=int(stats.kernels_total), status=int(stats.status),
                          logits=logits[:n] if logits is not None else None)
