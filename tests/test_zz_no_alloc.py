"""The allocation-free step (``fav_step_static``) against ``fav_step`` on a B200.

``fav_step_static`` exists for callers that cannot allocate device memory
while decoding (a real-time audio callback must not call cudaMalloc, which can
synchronise the device and block; some hosts forbid allocation after
start-up). It runs the same kernels with the step's scratch in a static
device array, so its audio and advanced histories must equal ``fav_step``'s
exactly. Two calls in a row are checked: a fresh start and a continuation
from the history the first call wrote. This file is collected last and
creates everything it uses, so it passes alone in a fresh process or after
the other tests.
"""
import ctypes as ct

import numpy as np
import pytest
import torch

from fast_audiovae import _native, build
from fast_audiovae import weights as W

pytestmark = pytest.mark.gpu


def ptr(t):
    return ct.c_void_p(t.data_ptr())


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not build.LIBRARY.exists():
        build.build()
    lib = _native.load_library()
    assert lib.fav_device_supported()
    return lib


def test_static_step_matches_fav_step_twice(lib):
    """Two calls in a row at the largest accepted size (fresh, then carried),
    then a smaller carried call over a subset of the streams. The ``fav_step``
    arm's workspace is filled with NaN bytes before every call, so a step that
    read scratch it had not written would differ between the two arms."""
    plan = _native.Plan(W.seeded_weights(0))
    n_max = 8
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    pools = [torch.zeros(lib.fav_state_pool_bytes(n_max) // 4, device="cuda") for _ in range(2)]
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    calls = [(8, 2, 2), (8, 2, 1), (3, 1, 0)]  # (streams, frames, fresh / read-table bits)
    assert calls[0][0] * calls[0][1] == 16  # FAV_STATIC_MAX_FRAMES
    for call, (n, frames, bits) in enumerate(calls):
        codes = torch.tensor([(s << 2) | bits for s in range(n)], dtype=torch.int32, device="cuda")
        z = torch.from_numpy(np.concatenate([W.seeded_latents(50 + 10 * call + s, frames) for s in range(n)])).cuda()
        ws_bytes = lib.fav_step_workspace_bytes(n, frames)
        ws = torch.full((ws_bytes,), 0xFF, dtype=torch.uint8, device="cuda")
        audio = [torch.full((n, 1920 * frames), float("nan"), device="cuda") for _ in range(2)]
        status.zero_()
        _native.check(lib, lib.fav_step(plan.handle, ptr(pools[0]), n_max, ptr(codes), n, frames, ptr(z),
                                        ptr(audio[0]), ptr(ws), ws_bytes, ptr(status[0:1]), stream))
        _native.check(lib, lib.fav_step_static(plan.handle, ptr(pools[1]), n_max, ptr(codes), n, frames, ptr(z),
                                               ptr(audio[1]), ptr(status[1:2]), stream))
        torch.cuda.synchronize()
        assert status.tolist() == [0, 0]
        assert torch.isfinite(audio[1]).all()
        assert torch.equal(audio[0], audio[1]), call
        assert torch.equal(pools[0].view(torch.int32), pools[1].view(torch.int32)), call


def test_static_step_matches_fav_step_on_an_int8_plan(lib):
    """An int8 (W8A8) plan needs no scratch beyond a bf16 one: the static step
    equals fav_step bit for bit on it too (fresh, then carried)."""
    plan = _native.Plan(W.seeded_weights(0), precision=1)
    n, frames = 4, 2
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    pools = [torch.zeros(lib.fav_state_pool_bytes(n) // 4, device="cuda") for _ in range(2)]
    ws_bytes = lib.fav_plan_workspace_bytes(plan.handle, n, frames)
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    for call, bits in enumerate((2, 1)):
        codes = torch.tensor([(s << 2) | bits for s in range(n)], dtype=torch.int32, device="cuda")
        z = torch.from_numpy(np.concatenate([W.seeded_latents(90 + 10 * call + s, frames) for s in range(n)])).cuda()
        ws = torch.full((ws_bytes,), 0xFF, dtype=torch.uint8, device="cuda")
        audio = [torch.full((n, 1920 * frames), float("nan"), device="cuda") for _ in range(2)]
        status.zero_()
        _native.check(lib, lib.fav_step(plan.handle, ptr(pools[0]), n, ptr(codes), n, frames, ptr(z), ptr(audio[0]),
                                        ptr(ws), ws_bytes, ptr(status[0:1]), stream))
        _native.check(lib, lib.fav_step_static(plan.handle, ptr(pools[1]), n, ptr(codes), n, frames, ptr(z),
                                               ptr(audio[1]), ptr(status[1:2]), stream))
        torch.cuda.synchronize()
        assert status.tolist() == [0, 0]
        assert torch.equal(audio[0], audio[1]), call
        assert torch.equal(pools[0].view(torch.int32), pools[1].view(torch.int32)), call


def test_static_step_rejects_sizes_beyond_its_limit(lib):
    plan = _native.Plan(W.seeded_weights(0))
    pool = torch.zeros(lib.fav_state_pool_bytes(17) // 4, device="cuda")
    codes = torch.tensor([(s << 2) | 2 for s in range(17)], dtype=torch.int32, device="cuda")
    z = torch.zeros(17, 64, 1, device="cuda")
    audio = torch.zeros(17, 1920, device="cuda")
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = lib.fav_step_static(plan.handle, ptr(pool), 17, ptr(codes), 17, 1, ptr(z), ptr(audio), None, stream)
    assert st == 4  # FAV_SIZE_OVERFLOW
    assert b"static workspace limit" in lib.fav_last_error()
    assert lib.fav_step_static(plan.handle, ptr(pool), 17, ptr(codes), 8, 3, ptr(z), ptr(audio), None, stream) == 4
