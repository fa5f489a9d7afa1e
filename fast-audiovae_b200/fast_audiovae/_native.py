"""ctypes binding of ``libfav_cuda.so`` (declarations in ``include/fast_audiovae_cuda.h``).

Loading never falls back to anything: a missing or unloadable library raises.
"""
from __future__ import annotations

import ctypes as ct
import threading
from pathlib import Path

import numpy as np

from . import weights as W

LIBRARY = Path(__file__).resolve().parent / "libfav_cuda.so"
ABI_VERSION = 1
SLOT_FLOATS = 161856
SLOT_STRIDE_FLOATS = 2 * SLOT_FLOATS + 64
NUM_COEFFICIENTS = 188

STATUS = {0: "FAV_OK", 1: "FAV_INVALID_ARGUMENT", 2: "FAV_UNSUPPORTED", 3: "FAV_OVERLAP",
          4: "FAV_SIZE_OVERFLOW", 5: "FAV_DEVICE_ERROR", 6: "FAV_TIMEOUT"}

# Every symbol the header declares, with its ctypes signature.
_P = ct.c_void_p
SIGNATURES = {
    "fav_abi_version": ([], ct.c_int32),
    "fav_last_error": ([], ct.c_char_p),
    "fav_status_string": ([ct.c_int32], ct.c_char_p),
    "fav_device_supported": ([], ct.c_int32),
    "fav_host_device_pointer": ([ct.c_void_p, ct.POINTER(ct.c_void_p)], ct.c_int32),
    "fav_plan_create": ([ct.POINTER(ct.POINTER(ct.c_float)), ct.c_int32, ct.c_int32, ct.POINTER(_P)], ct.c_int32),
    "fav_plan_destroy": ([_P], None),
    "fav_plan_bytes": ([_P], ct.c_size_t),
    "fav_state_pool_bytes": ([ct.c_int32], ct.c_size_t),
    "fav_step_workspace_bytes": ([ct.c_int32, ct.c_int32], ct.c_size_t),
    "fav_step": ([_P, _P, ct.c_int32, _P, ct.c_int32, ct.c_int32, _P, _P, _P, ct.c_size_t, _P, _P], ct.c_int32),
    "fav_debug_step_unfused": ([_P, _P, ct.c_int32, _P, ct.c_int32, ct.c_int32, _P, _P, _P, ct.c_size_t, _P, _P],
                               ct.c_int32),
    "fav_step_static": ([_P, _P, ct.c_int32, _P, ct.c_int32, ct.c_int32, _P, _P, _P, _P], ct.c_int32),
    "fav_batch_workspace_bytes": ([ct.c_int32, ct.c_int32], ct.c_size_t),
    "fav_plan_workspace_bytes": ([_P, ct.c_int32, ct.c_int32], ct.c_size_t),
    "fav_plan_batch_workspace_bytes": ([_P, ct.c_int32, ct.c_int32], ct.c_size_t),
    "fav_plan_precision": ([_P], ct.c_int32),
    "fav_decode_batch": ([_P, _P, ct.c_int32, ct.c_int32, ct.c_int32, _P, _P, ct.c_size_t, _P, _P], ct.c_int32),
    "fav_step_profile": ([_P, _P, ct.c_int32, _P, ct.c_int32, ct.c_int32, _P, _P, _P, ct.c_size_t, _P,
                          ct.POINTER(ct.c_float), _P], ct.c_int32),
    "fav_debug_step_layers": ([_P, _P, ct.c_int32, _P, ct.c_int32, ct.c_int32, _P, _P, ct.c_size_t, _P,
                               ct.c_int32, ct.POINTER(ct.c_void_p), _P], ct.c_int32),
    "fav_debug_step_gated": ([_P, _P, ct.c_int32, _P, ct.c_int32, ct.c_int32, _P, _P, _P, ct.c_size_t, _P,
                              ct.c_int32, ct.c_uint32, _P, _P], ct.c_int32),
    "fav_test_gemm": ([_P, ct.c_int32, ct.c_int32, _P, ct.c_int32, ct.c_int32, _P, _P], ct.c_int32),
    "fav_test_sine": ([_P, ct.c_int32, _P, _P], ct.c_int32),
}

_lock = threading.Lock()
_lib = None


class NativeError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status


def load_library(path=None):
    """Load (once) and type the CUDA library; raises if it is absent or mismatched."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        target = Path(path) if path else LIBRARY
        if not target.is_file():
            raise RuntimeError(f"CUDA decoder library {target} is not built; run fast_audiovae.build")
        lib = ct.CDLL(str(target))
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        if lib.fav_abi_version() != ABI_VERSION:
            raise RuntimeError("CUDA decoder ABI version mismatch")
        if path is None:
            _lib = lib
        return lib


def check(lib, status):
    if status != 0:
        raise NativeError(status, lib.fav_last_error().decode(errors="replace"))


def coefficient_list(weights):
    """The 188 coefficient arrays in the C ABI's canonical order (contiguous fp32)."""
    W.validate_weights(weights)
    names = list(W.weight_shapes())
    assert len(names) == NUM_COEFFICIENTS
    return [np.ascontiguousarray(weights[n], dtype=np.float32) for n in names]


class Plan:
    """Owns an ``fav_plan`` (immutable packed weights on the current device)."""

    def __init__(self, weights, precision=0):
        self.lib = load_library()
        arrays = coefficient_list(weights)
        self._keep = arrays
        ptrs = (ct.POINTER(ct.c_float) * len(arrays))(*[a.ctypes.data_as(ct.POINTER(ct.c_float)) for a in arrays])
        handle = ct.c_void_p()
        check(self.lib, self.lib.fav_plan_create(ptrs, len(arrays), precision, ct.byref(handle)))
        self.handle = handle
        self._keep = None

    @property
    def device_bytes(self):
        return int(self.lib.fav_plan_bytes(self.handle))

    def close(self):
        if getattr(self, "handle", None):
            self.lib.fav_plan_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
