"""Loaders for the real reference code, used only to pin the oracle (test infrastructure).

* ``reference_decoder(weights)``: the reference's own explicit fp32 decoder
  ``MPSModel`` (``src/fast_audiovae/mps_decoder.py:156-325``) on ``device='cpu'``,
  assembled from a coefficient dict through its public module constructors
  (``_Snake``, ``_Pointwise``, ``_CausalConv1d``, ``_CausalTranspose1d``,
  ``_Residual``, ``_Stage``; ``from_onnx`` is skipped because the pinned export is
  absent). The package ``__init__`` imports onnxruntime, so ``mps_decoder.py`` and
  ``assets.py`` are loaded by file path under a stub package.
* ``precision_library()`` / ``native_library()``: ctypes handles on the reference's
  C sources compiled by ``oracle/Makefile`` into ``oracle/_ref``.

The reference tree exists only in the build container; callers skip when
``REFERENCE_ROOT`` is missing. ``REFERENCE_ROOT`` is the one place that says
where it is mounted (``$FAST_AUDIOVAE_REFERENCE`` overrides it); the golden
generator and the build read it from here.
"""
from __future__ import annotations

import ctypes as ct
import importlib.util
import os
import sys
import types
from pathlib import Path

import numpy as np

REFERENCE_ROOT = Path(os.environ.get("FAST_AUDIOVAE_REFERENCE", "/root/reference"))
REF_LIB_DIR = Path(__file__).resolve().parent / "_ref"


def reference_available():
    return (REFERENCE_ROOT / "src/fast_audiovae/mps_decoder.py").is_file()


def _load_mps_decoder():
    name = "_fav_reference_pkg"
    if name + ".mps_decoder" in sys.modules:
        return sys.modules[name + ".mps_decoder"]
    src = REFERENCE_ROOT / "src/fast_audiovae"
    package = types.ModuleType(name)
    package.__path__ = [str(src)]
    sys.modules[name] = package
    for module in ("assets", "mps_decoder"):
        spec = importlib.util.spec_from_file_location(f"{name}.{module}", src / f"{module}.py")
        loaded = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = loaded
        spec.loader.exec_module(loaded)
    return sys.modules[name + ".mps_decoder"]


def reference_module():
    if not reference_available():
        raise FileNotFoundError("reference sources are not present")
    return _load_mps_decoder()


def reference_decoder(weights):
    """Build the reference ``MPSModel`` (fp32, CPU) from a coefficient dict."""
    m = reference_module()
    w = {k: np.ascontiguousarray(v, dtype=np.float32) for k, v in weights.items()}
    stem = m._CausalConv1d(w["stem.weight"], w["stem.bias"], groups=64)
    pw = m._Pointwise(w["pointwise.weight"], w["pointwise.bias"])
    stages = []
    for i, stride in enumerate((8, 6, 5, 2, 2, 2)):
        p = f"stage{i}."
        before = m._Snake(w[p + "snake.alpha"], w[p + "snake.reciprocal"])
        transpose = m._CausalTranspose1d(w[p + "transpose.weight"], w[p + "transpose.bias"],
                                         stride=stride, paired=(i == 0))
        residuals = []
        for j, d in enumerate((1, 3, 9)):
            r = f"{p}residual{j}."
            cout = w[r + "depthwise.weight"].shape[0]
            residuals.append(m._Residual(
                m._Snake(w[r + "pre.alpha"], w[r + "pre.reciprocal"]),
                m._CausalConv1d(w[r + "depthwise.weight"], w[r + "depthwise.bias"], dilation=d, groups=cout),
                m._Snake(w[r + "post.alpha"], w[r + "post.reciprocal"]),
                m._Pointwise(w[r + "pointwise.weight"], w[r + "pointwise.bias"])))
        stages.append(m._Stage(w[p + "scale"], w[p + "offset"], before, transpose, residuals))
    final_snake = m._Snake(w["final.snake.alpha"], w["final.snake.reciprocal"])
    final_conv = m._CausalConv1d(w["final.weight"], w["final.bias"])
    model = m.MPSModel(stem, pw, stages, final_snake, final_conv)
    assert len(model.state_shapes) == 26 and model.state_bytes == 647424
    return model


def _library(name):
    path = REF_LIB_DIR / name
    if not path.is_file():
        raise FileNotFoundError(f"{path} is not built; run make -C oracle ref")
    return ct.CDLL(str(path))


def precision_library():
    """ctypes handle on the reference int8 core (``precision.cpp``, scalar backend 0)."""
    lib = _library("libprecision_ref.so")
    P = ct.POINTER(ct.c_float)
    for name, args, res in [
            ("ip_abi", [], ct.c_int), ("ip_last_error", [], ct.c_char_p),
            ("ip_create", [ct.c_int, ct.c_int, P, ct.c_int, ct.c_int], ct.c_void_p),
            ("ip_prepare", [ct.c_void_p, P, ct.c_int], ct.c_void_p),
            ("ip_run_rows", [ct.c_void_p, ct.c_void_p, P, ct.c_int, ct.c_int], ct.c_int),
            ("ip_destroy_plan", [ct.c_void_p], None), ("ip_destroy_input", [ct.c_void_p], None)]:
        fn = getattr(lib, name)
        fn.argtypes, fn.restype = args, res
    assert lib.ip_abi() == 1
    return lib


def precision_matmul(w, x, mode=8):
    """``y = W8A8(w, x)`` through the compiled reference core (backend 0)."""
    lib = precision_library()
    P = ct.POINTER(ct.c_float)
    w = np.ascontiguousarray(w, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    m, k = w.shape
    t = x.shape[1]
    plan = lib.ip_create(m, k, w.ctypes.data_as(P), mode, 0)
    if not plan:
        raise RuntimeError(lib.ip_last_error().decode())
    try:
        inp = lib.ip_prepare(plan, x.ctypes.data_as(P), t)
        if not inp:
            raise RuntimeError(lib.ip_last_error().decode())
        try:
            y = np.full((m, t), np.nan, np.float32)
            if lib.ip_run_rows(plan, inp, y.ctypes.data_as(P), 0, m):
                raise RuntimeError(lib.ip_last_error().decode())
            return y
        finally:
            lib.ip_destroy_input(inp)
    finally:
        lib.ip_destroy_plan(plan)


def native_library():
    """ctypes handle on the reference x86 elementwise kernels (scalar libm build)."""
    lib = _library("libncc_ref.so")
    P = ct.POINTER(ct.c_float)
    i64, i32 = ct.c_int64, ct.c_int32
    lib.ncc_abi_version.restype = ct.c_uint32
    lib.ncc_snake_f32.argtypes = [P, P, P, P, i64, i64, i64, i32, i32]
    lib.ncc_snake_f32.restype = i32
    lib.ncc_dw7_f32_ex.argtypes = [P, P, P, P, P, P, P, i64, i64, i64, i32, i32, i32]
    lib.ncc_dw7_f32_ex.restype = i32
    lib.ncc_snake_dw7_snake_f32.argtypes = [P, P, P, P, P, P, P, P, i64, i64, i64, i32, i32, i32]
    lib.ncc_snake_dw7_snake_f32.restype = i32
    lib.ncc_bias_residual_f32.argtypes = [P, P, P, P, i64, i64, i64, i32, i32]
    lib.ncc_bias_residual_f32.restype = i32
    return lib
