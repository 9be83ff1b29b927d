"""ctypes binding of the C ABI in ``include/bifrost_b200.h`` (library ``lib/libbifrost_b200.so``).

The library is loaded once per process.  There is no fallback: if it is missing or no sm_100
device is present, the calls raise.  ``call(name, *args)`` raises ``RuntimeError`` with
``bf_strerror(code)`` for any non-zero status, mirroring the reference's exception-based errors.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libbifrost_b200.so"

_P = ctypes.c_void_p
_I = ctypes.c_int
_Z = ctypes.c_size_t
_L = ctypes.c_longlong

# name -> (argtypes); every entry point returns int (status) unless listed in _RESTYPE
SIGNATURES = {
    "bf_strerror": [_I],
    "bf_last_cuda_error": [],
    "bf_abi_version": [],
    "bf_device_error": [_P, _P],
    "bf_selftest_wait_timeout": [ctypes.c_uint, _P],
    "bf_stage_events": [_P, _I],
    "bf_gdn_decode_step": [_P, _P, _P, _I, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "bf_layer_weights_bytes": [_I, _I, _I, _I],
    "bf_prepare_layer_weights": [_P, _P, _P, _P, _I, _I, _I, _I, _P, _Z, _P],
    "bf_mem_inputs": [_P, _P, _P, _P, _P, ctypes.c_longlong, _I, _I, _P, _P, _P, _P, _P, _P],
    "bf_layer_decode_workspace": [_I, _I, _I, _I, _I],
    "bf_bifrost_layer_decode": [_P, _P, _P, _P, _P, _P, _P, _P, _I, _P, _I, _P, _P, _P, _Z, _P],
    "bf_bifrost_layer_decode_noalloc": [_P, _P, _P, _P, _P, _P, _P, _P, _I, _P, _I, _P, _P, _P],
    "bf_gdn_chunk_workspace": [_I, _I, _I, _I, _I, _I],
    "bf_gdn_chunk_fwd": [_P, _I, _P, _I, _P, _I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _Z, _P],
    "bf_gdn_bwd_workspace": [_I, _I, _I, _I, _I],
    "bf_gdn_bwd": [_P] * 14 + [_I, _I, _I, _I, _I, _P, _Z, _P],
    "bf_window_workspace": [_I, _I, _I, _I],
    "bf_window_attn_fwd": [_P, _P, _P, _L, _L, _L, _P, _P, _I, _L, _L, _L, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P,
                           _Z, _P],
    "bf_layer_prefill_workspace": [_I, _I, _I, _I, _I, _I, _I],
    "bf_layer_prefill_sp_workspace": [_I, _I, _I, _I, _I, _I, _I],
    "bf_bifrost_layer_prefill": [_P, _P, _P, _P, _P, _P, _P, _L, _I, _I, _P, _P, _P, _I, _I, _P, _P, _P, _Z, _P],
    "bf_attn_prologue": [_P, _P, _P, _P, _P, _I, ctypes.c_float, _L, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P],
    "bf_attn_epilogue": [_P, _P, _I, _I, _I, _I, _I, _P, _P],
    "bf_gdn_segment_workspace": [_I, _I, _I, _I],
    "bf_gdn_segment_transform": [_P, _I, _P, _I, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _Z, _P],
    "bf_gdn_apply_prefix": [_P, _P, _I, _P, _P, _I, _I, _I, _P],
    "bf_bifrost_layer_prefill_sp": [_P, _P, _P, _P, _P, _P, _P, _L, _I, _I, _P, _P, _P, _I, _I, _P, _P, _P, _P, _P,
                                    _Z, _P],
    "bf_ret_summarize": [_P, _L, _I, _I, _I, _I, _I, _I, _I, _P, _P, _L, _P],
    "bf_ret_decode_workspace": [_I, _I, _I, _I, _I, _I, _I, _I, _I],
    "bf_ret_decode": [_P, _P, _P, _L, _P, _P, _L, _I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _Z, _P],
    "bf_llama_state_floats": [_I, _I, _I, _I],
    "bf_llama_state_pack": [_P, _P, _I, _I, _I, _I, _I, _P, _L, _P],
    "bf_llama_state_unpack": [_P, _L, _P, _I, _I, _I, _I, _I, _P, _P],
}
_RESTYPE = {"bf_strerror": ctypes.c_char_p, "bf_last_cuda_error": ctypes.c_char_p, "bf_layer_weights_bytes": _Z, "bf_layer_decode_workspace": _Z,
            "bf_gdn_chunk_workspace": _Z, "bf_window_workspace": _Z, "bf_layer_prefill_workspace": _Z,
            "bf_layer_prefill_sp_workspace": _Z,
            "bf_gdn_segment_workspace": _Z, "bf_llama_state_floats": _Z,
            "bf_ret_decode_workspace": _Z, "bf_gdn_bwd_workspace": _Z}

_lock = threading.Lock()
_lib = None


class BifrostError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, name: str, code: int, msg: str):
        super().__init__(f"{name}: {msg} (status {code})")
        self.code = code


def load() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH} is missing: run `python -m heimdall_b200.build` "
                                   "(there is no CPU fallback)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, argt in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argt
                fn.restype = _RESTYPE.get(name, _I)
            _lib = lib
    return _lib


def strerror(code: int) -> str:
    return load().bf_strerror(code).decode()


def size(name: str, *args) -> int:
    """Call a size query (returns size_t)."""
    return int(getattr(load(), name)(*args))


def call(name: str, *args) -> None:
    rc = getattr(load(), name)(*args)
    if rc != 0:
        msg = strerror(rc)
        if rc == 5:   # BF_ERR_CUDA: add the CUDA error behind it
            msg += ": " + load().bf_last_cuda_error().decode()
        raise BifrostError(name, rc, msg)


def device_error(stream: int = 0):
    """(word, block_x, block_yz, thread) of the first device-side wait that gave up since the last read."""
    w = (ctypes.c_uint * 4)()
    call("bf_device_error", w, stream)
    return tuple(int(x) for x in w)


def declared_symbols() -> list:
    """Entry points declared in include/bifrost_b200.h (parsed from the header text)."""
    import re
    hdr = (Path(__file__).resolve().parents[1] / "include" / "bifrost_b200.h").read_text()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(bf_\w+)\s*\(", hdr, flags=re.M)))
