"""Batched serving over the C ABI: B sequences in lockstep on one GPU, or one
rank of a tensor-parallel group over KV-head groups.

The reference serves long-context batches by running each sequence through
CachedForwardPlan::prepare_device_generation / start_sequence
(src/inference/executor.cpp:1482-1716) one after another.  `Server` runs the
batch together: every weight read serves all B rows, and with tp_size > 1
each GPU holds 1/tp_size of the query heads, KV heads, MLP columns and
vocabulary-head rows, the o_proj and down_proj partial sums meeting in an
all-reduce and the logits in an all-gather.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import check, lib
from .engine import Qwen3Config, Settings


@dataclass
class ServeResult:
    tokens: np.ndarray            # [steps][batch]
    logits: np.ndarray | None     # [steps][batch][V] BF16 bits
    decode_ms: float
    prefill_ms: float             # device time of the last prefill (prompt passes + first selections)
    kernels_per_decode_step: int


class Server:
    def __init__(self, config: Qwen3Config, batch: int, capacity: int, chunk_rows: int = 1024, device: int = 0,
                 tp_rank: int = 0, tp_size: int = 1):
        self.config = config
        self.batch = batch
        self.tp_rank, self.tp_size = tp_rank, tp_size
        h = C.c_void_p()
        check(lib().dl_serve_create(C.byref(config.c()), device, batch, capacity, chunk_rows, tp_rank, tp_size,
                                    C.byref(h)))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().dl_serve_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def nccl_id() -> bytes:
        buf = (C.c_ubyte * 128)()
        check(lib().dl_serve_nccl_id(buf))
        return bytes(buf)

    def connect(self, nccl_id: bytes) -> None:
        buf = (C.c_ubyte * 128).from_buffer_copy(nccl_id)
        check(lib().dl_serve_connect(self._h, buf))

    def ipc_handle(self) -> bytes:
        buf = (C.c_ubyte * 64)()
        check(lib().dl_serve_ipc_handle(self._h, buf))
        return bytes(buf)

    def connect_peers(self, handles: bytes) -> None:
        buf = (C.c_ubyte * len(handles)).from_buffer_copy(handles)
        check(lib().dl_serve_connect_peers(self._h, buf))

    def init_random(self, seed: int, sigma: float = 0.02) -> None:
        check(lib().dl_serve_init_random(self._h, seed, sigma))

    def set_sampler_engine(self, engine: int) -> None:
        """Draw source of later prefills' sequences (DL_RNG_*)."""
        check(lib().dl_serve_set_sampler_engine(self._h, engine))

    def set_capture(self, layer: int) -> None:
        """Block `layer`'s output rows of every sequence and position; -1 off."""
        check(lib().dl_serve_set_capture(self._h, layer))

    def read_capture(self, sequence: int, first: int, count: int) -> np.ndarray:
        out = np.empty((count, self.config.hidden), np.uint16)
        check(lib().dl_serve_read_capture(self._h, sequence, first, count, out.ctypes.data_as(_lib.u16p)))
        return out

    def set_steering(self, layer: int, first_position: int = 0, strength: float = 0.0, direction=None,
                     sequences=(), source_sequence: int = -1, source_position: int = 0) -> None:
        """Fixed-strength steering of every position >= first_position at
        block `layer` for the listed sequences: h' = round(h + beta*u).
        beta = strength, or strength * ||h|| of sequence source_sequence's
        block output at source_position (computed in the prompt pass).
        layer < 0 turns it off."""
        if layer < 0:
            check(lib().dl_serve_set_steering(self._h, -1, 0, 0.0, None, None, -1, 0))
            return
        u = np.ascontiguousarray(direction, np.float32)
        if u.size != self.config.hidden:
            raise ValueError("steering direction must have the hidden width")
        mask = np.zeros(self.batch, np.uint8)
        mask[list(sequences)] = 1
        check(lib().dl_serve_set_steering(self._h, layer, first_position, strength,
                                          u.ctypes.data_as(C.POINTER(C.c_float)),
                                          mask.ctypes.data_as(C.POINTER(C.c_uint8)), source_sequence,
                                          source_position))

    def set_step_fusion(self, on: bool) -> None:
        """Fused decode step (default) or separate kernels; the same bits."""
        check(lib().dl_serve_set_step_fusion(self._h, 1 if on else 0))

    def steering_strength(self) -> float:
        b = C.c_float()
        check(lib().dl_serve_steering_strength(self._h, C.byref(b)))
        return b.value

    def set_tensor(self, index: int, full_bits: np.ndarray) -> None:
        b = np.ascontiguousarray(full_bits, dtype=np.uint16)
        check(lib().dl_serve_set_tensor(self._h, index, b.ctypes.data, b.nbytes))

    def slice_shape(self, index: int) -> tuple:
        r, c, r0, c0 = C.c_size_t(), C.c_size_t(), C.c_size_t(), C.c_size_t()
        check(lib().dl_serve_slice_shape(self._h, index, C.byref(r), C.byref(c), C.byref(r0), C.byref(c0)))
        return r.value, c.value, r0.value, c0.value

    def get_tensor(self, index: int) -> np.ndarray:
        rows, cols, _, _ = self.slice_shape(index)
        out = np.empty((rows, cols), np.uint16)
        check(lib().dl_serve_get_tensor(self._h, index, out.ctypes.data, out.nbytes))
        return out

    @property
    def position(self) -> int:
        return int(lib().dl_serve_position(self._h))

    def prefill(self, prompts, settings: Settings | None = None, seed: int = 0) -> np.ndarray:
        """prompts [batch][P] token ids; returns each sequence's first token."""
        settings = settings or Settings()
        p = np.ascontiguousarray(prompts, dtype=np.uint32)
        if p.ndim != 2 or p.shape[0] != self.batch:
            raise ValueError("prompts must be [batch][prompt_len]")
        first = np.zeros(self.batch, np.uint32)
        s = settings.c()
        check(lib().dl_serve_prefill(self._h, p.ctypes.data_as(_lib.u32p), p.shape[1], C.byref(s), seed,
                                     first.ctypes.data_as(_lib.u32p)))
        return first

    def decode(self, steps: int, want_logits: bool = False) -> ServeResult:
        tokens = np.zeros((steps, self.batch), np.uint32)
        logits = np.empty((steps, self.batch, self.config.vocabulary), np.uint16) if want_logits else None
        stats = _lib.ServeStats()
        check(lib().dl_serve_decode(self._h, steps, tokens.ctypes.data_as(_lib.u32p),
                                    logits.ctypes.data_as(_lib.u16p) if logits is not None else None,
                                    C.byref(stats)))
        return ServeResult(tokens, logits, stats.decode_ms, stats.prefill_ms, int(stats.kernels_per_decode_step))


# Per-block tensor roles (engine order) and how tensor parallelism cuts them:
# "rows" = output features of a column-parallel projection, "cols" = input
# features of a row-parallel one, None = replicated.
_ROLE_CUT = {0: None, 1: ("rows", "q"), 2: ("rows", "kv"), 3: ("rows", "kv"), 4: None, 5: None, 6: ("cols", "q"),
             7: None, 8: ("rows", "mlp"), 9: ("rows", "mlp"), 10: ("cols", "mlp")}


def tp_slices(config: Qwen3Config, rank: int, size: int) -> list:
    """(rows, cols, r0, c0) of every tensor (engine order) that rank `rank`
    of a tensor-parallel group of `size` holds: query heads, KV heads, MLP
    columns and vocabulary-head rows in `size` equal contiguous slices (the
    layout Server uses)."""
    if (size < 1 or not 0 <= rank < size or config.kv_heads % size or config.mlp_width % size
            or config.vocabulary % size):
        raise ValueError("tensor-parallel size must divide the KV heads, the MLP width and the vocabulary")
    d = config.head_width
    width = {"q": config.query_heads * d // size, "kv": config.kv_heads * d // size, "mlp": config.mlp_width // size}
    shapes = [(config.vocabulary, config.hidden), (1, config.hidden), (config.vocabulary, config.hidden)]
    full_q, full_kv = config.query_heads * d, config.kv_heads * d
    per_block = [(1, config.hidden), (full_q, config.hidden), (full_kv, config.hidden), (full_kv, config.hidden),
                 (1, d), (1, d), (config.hidden, full_q), (1, config.hidden), (config.mlp_width, config.hidden),
                 (config.mlp_width, config.hidden), (config.hidden, config.mlp_width)]
    out = [(r, c, 0, 0) for r, c in shapes]
    vl = config.vocabulary // size
    out[2] = (vl, config.hidden, rank * vl, 0)  # vocabulary head: row slices
    for _ in range(config.layers):
        for role, (r, c) in enumerate(per_block):
            cut = _ROLE_CUT[role]
            if cut is None:
                out.append((r, c, 0, 0))
            elif cut[0] == "rows":
                w = width[cut[1]]
                out.append((w, c, rank * w, 0))
            else:
                w = width[cut[1]]
                out.append((r, w, 0, rank * w))
    return out


def connect_group(server, dist, make_id=Server.nccl_id, peers: bool = True) -> bytes:
    """Connect a tensor-parallel group over the torch.distributed process
    group (any backend): rank 0's NCCL id reaches every rank and every rank
    connects with it; then (peers) the ranks swap CUDA IPC handles of their
    peer all-reduce buffers, in rank order."""
    obj = [make_id() if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    server.connect(obj[0])
    if peers:
        handles = [None] * dist.get_world_size()
        dist.all_gather_object(handles, server.ipc_handle())
        server.connect_peers(b"".join(handles))
    return obj[0]
