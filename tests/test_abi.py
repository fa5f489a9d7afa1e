"""The C-ABI library: loads on any machine, exports every declared symbol (CPU).

No compute call is made here; only host-side entry points that need no GPU.
"""
import ctypes as ct
import re
from pathlib import Path

import pytest

from fast_audiovae import _native, build

HEADER = Path(__file__).resolve().parent.parent / "include" / "fast_audiovae_cuda.h"


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _native.load_library()


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"FAV_API\s+[\w\s\*]+?\b(fav_\w+)\s*\(", text)))


def test_header_declares_the_bound_symbols():
    assert declared_symbols() == sorted(_native.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_library_exports_nothing_else():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", str(build.LIBRARY)], capture_output=True, text=True)
    if out.returncode:
        pytest.skip("nm unavailable")
    exported = sorted({line.split()[-1] for line in out.stdout.splitlines() if " T " in line and "fav_" in line})
    assert exported == declared_symbols()


def test_abi_version_and_sizes(lib):
    assert lib.fav_abi_version() == 1
    assert lib.fav_state_pool_bytes(3) == 3 * (2 * 647424 + 256)
    assert lib.fav_state_pool_bytes(0) == 0
    assert lib.fav_step_workspace_bytes(2, 3) == 2 * 3 * 6 * 61440 * 4
    assert lib.fav_step_workspace_bytes(0, 3) == 0
    assert lib.fav_batch_workspace_bytes(2, 4) == 2 * 4 * 6 * 61440 * 4 + 2 * (2 * 647424 + 256)
    assert lib.fav_status_string(6) == b"device wait timed out"


def test_plan_create_rejects_bad_arguments_before_device_use(lib):
    handle = ct.c_void_p()
    assert lib.fav_plan_create(None, 188, 0, ct.byref(handle)) == 1
    assert b"188" in lib.fav_last_error()
    arrays = (ct.POINTER(ct.c_float) * 3)()
    assert lib.fav_plan_create(arrays, 3, 0, ct.byref(handle)) == 1
    assert not handle.value


def test_step_rejects_bad_arguments(lib):
    assert lib.fav_step(None, None, 0, None, 1, 1, None, None, None, 0, None, None) == 1
    assert b"plan" in lib.fav_last_error()


def test_library_is_sm100a_only():
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.NVCC_FLAGS)
