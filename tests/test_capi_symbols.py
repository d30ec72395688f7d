"""The C-ABI library loads without a GPU and exports every symbol the public
header declares; host-only entry points answer without touching a device."""
import ctypes as C

import pytest

import dolittle_b200 as dl
from dolittle_b200 import _lib


def test_library_exports_every_header_symbol():
    L = dl.lib()
    names = dl.header_symbols()
    assert len(names) >= 35
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    # The binding table covers the whole header too.
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)


def test_host_only_entry_points():
    L = dl.lib()
    assert b"sm_100a" in L.dl_version()
    cfg = dl.QWEN3_8B
    assert cfg.tensor_count() == 3 + 11 * 36
    assert cfg.tensor_shape(0) == (151936, 4096)
    assert cfg.tensor_shape(3 + 1) == (4096, 4096)       # block 0 q
    assert cfg.tensor_shape(3 + 2) == (1024, 4096)       # block 0 k
    assert cfg.tensor_shape(3 + 10) == (4096, 12288)     # block 0 down
    assert L.dl_attention_workspace_bytes(1, 32, 1024) == 32 * 1024 * 4
    assert L.dl_sampler_required_bytes(151936) > 151936 * 24


def test_invalid_arguments_are_rejected_before_any_launch():
    L = dl.lib()
    # FP32 storage is not part of the product: rejected, never converted.
    assert L.dl_projection(dl.DL_F32, None, None, None, 1, 8, 8, None, None) == _lib.DL_UNSUPPORTED
    assert L.dl_projection(dl.DL_BF16, None, None, None, 1, 8, 8, None, None) == _lib.DL_INVALID_ARGUMENT
    assert b"null" in L.dl_last_error()
    # The draw source is chosen from the two known engines only.
    assert L.dl_sampler_set_engine(None, dl.DL_RNG_PHILOX4X32_10) == _lib.DL_INVALID_ARGUMENT
    assert L.dl_engine_set_sampler_engine(None, 5) == _lib.DL_INVALID_ARGUMENT
    assert L.dl_direction(dl.DL_BF16, None, None, 8, None, None, None) == _lib.DL_INVALID_ARGUMENT
    with pytest.raises(dl.DolittleError):
        dl.Qwen3Config().tensor_shape(10_000)


def test_package_has_no_fallback_path():
    """Importing the engine never routes through the oracle or a CPU path."""
    import dolittle_b200.engine as eng
    src = open(eng.__file__).read() + open(_lib.__file__).read()
    assert "oracle" not in src and "numpy.dot" not in src
