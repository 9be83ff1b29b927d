"""CPU-side checks of the C ABI: the library loads without a GPU and exports every declared symbol."""
import ctypes

import pytest

from heimdall_b200 import _lib


def test_library_loads_and_exports_header_symbols():
    lib = _lib.load()
    names = _lib.declared_symbols()
    assert len(names) >= 5
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/bifrost_b200.h but not exported"
    assert set(names) == set(_lib.SIGNATURES), "ctypes signature table and header disagree"


def test_status_strings_and_version():
    assert _lib.strerror(0) == "ok"
    assert "workspace" in _lib.strerror(4)
    assert _lib.load().bf_abi_version() >= 1


def test_size_queries_need_no_device():
    assert _lib.size("bf_layer_weights_bytes", 24, 4, 256, 5120) >= 28 * 256 * 256 * 2
    assert _lib.size("bf_layer_decode_workspace", 64, 24, 4, 256, 2048) > 0


def test_invalid_arguments_rejected_before_launch():
    # null pointers are rejected without touching a device
    with pytest.raises(_lib.BifrostError) as e:
        _lib.call("bf_gdn_decode_step", 0, 0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 256, 0)
    assert e.value.code == 1
    with pytest.raises(_lib.BifrostError):
        _lib.call("bf_prepare_layer_weights", 0, 0, 0, 0, 24, 4, 256, 5120, 0, 0, 0)


def test_selftest_rejects_bad_limits_without_a_device():
    for bad in (0, 2_000_000):
        with pytest.raises(_lib.BifrostError) as e:
            _lib.call("bf_selftest_wait_timeout", bad, 0)
        assert e.value.code == 1


def test_noalloc_scratch_bound_pinned():
    """The allocation-free decode entry point's fixed scratch (16 MiB) holds the Bifrost geometry's decode
    workspace for 64 sequences at W = 2048 (the documented limit) and not for 128."""
    assert _lib.size("bf_layer_decode_workspace", 64, 24, 4, 256, 2048) <= 16 << 20
    assert _lib.size("bf_layer_decode_workspace", 128, 24, 4, 256, 2048) > 16 << 20
