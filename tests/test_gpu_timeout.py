"""Bounded waits that run out, on a B200 (``-m gpu``).

Every mbarrier wait in the GEMM engine and the fused stage kernels is bounded; when one runs out the
kernel drains the copies and MMAs it started, records a timeout code in the
caller's status word and returns, so the CUDA context stays usable. The
reference's streaming contract (``src/fast_audiovae/gpu.py:216-225``) is that
a failed step leaves the stream's history as it was. ``fav_debug_step_gated``
makes one engine (or fused stage) launch wait for a device flag that nothing sets, with a
short poll limit on every wait of that launch: nothing faults or hangs, the
status word reports the timeout, and the next ordinary step from the same
committed history gives the same audio as a run that never failed.
"""
import ctypes as ct

import numpy as np
import pytest
import torch

from fast_audiovae import _native, build
from fast_audiovae import weights as W

pytestmark = pytest.mark.gpu

TIMEOUT_CODES = {0x101, 0x102, 0x103, 0x104, 0x107}
S, F = 4, 1


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


@pytest.fixture(scope="module")
def plan(lib):
    return _native.Plan(W.seeded_weights(0))


class Run:
    """One history pool driven by ordinary and gated steps."""

    def __init__(self, lib, plan):
        self.lib, self.plan = lib, plan
        self.pool = torch.zeros(lib.fav_state_pool_bytes(S) // 4, device="cuda")
        self.ws_bytes = lib.fav_plan_workspace_bytes(plan.handle, S, F)
        self.ws = torch.full((self.ws_bytes,), 0xFF, dtype=torch.uint8, device="cuda")
        self.status = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
        self.steps = 0

    def codes(self):
        fresh = 2 if self.steps == 0 else 0
        return torch.tensor([(s << 2) | fresh | (self.steps & 1) for s in range(S)], dtype=torch.int32,
                            device="cuda")

    def latents(self, step):
        return torch.from_numpy(np.concatenate([W.seeded_latents(300 + s, 8)[..., step:step + F]
                                                for s in range(S)])).cuda()

    def step(self, gated_layer=None, gate=None):
        """Runs the next step; returns (audio, status). Commits (flips the read table) only on success."""
        audio = torch.full((S, 1920 * F), float("nan"), device="cuda")
        self.status.zero_()
        # Held until the step has finished: a device pointer taken from a tensor
        # that is then freed may be handed to the next allocation on this stream.
        codes, z = self.codes(), self.latents(self.steps)
        args = (self.plan.handle, ptr(self.pool), S, ptr(codes), S, F, ptr(z), ptr(audio), ptr(self.ws),
                self.ws_bytes, ptr(self.status))
        if gated_layer is None:
            _native.check(self.lib, self.lib.fav_step(*args, self.stream))
        else:
            _native.check(self.lib, self.lib.fav_debug_step_gated(*args, gated_layer, 1000, ptr(gate), self.stream))
        torch.cuda.synchronize()
        status = int(self.status.item()) & 0xFFFFFFFF
        if status == 0:
            self.steps += 1
        return audio.cpu(), status


def committed_windows(pool, read_table=0):
    """Every stream's read head table and the 26 history windows it names (ring
    rows [head, head + H) modulo 2H of each history, channels last)."""
    slots = pool.view(S, _native.SLOT_STRIDE_FLOATS).cpu()
    parts = []
    for slot in slots:
        heads = slot[2 * _native.SLOT_FLOATS:].view(torch.int32)[32 * read_table:32 * read_table + 32]
        parts.append(heads.view(torch.float32))
        off = 0
        for index, (_, (_, channels, rows)) in enumerate(W.state_shapes().items()):
            ring = slot[2 * off:2 * off + 2 * rows * channels].view(2 * rows, channels)
            parts.append(ring[(int(heads[index]) + torch.arange(rows)) % (2 * rows)].reshape(-1))
            off += rows * channels
    return torch.cat(parts).view(torch.int32)  # bit patterns: packed history rows may read as NaN


@pytest.mark.parametrize("layer", [0, 1, 2, 9, 10, 14, 20])
def test_gated_launch_times_out_and_history_survives(lib, plan, layer):
    """Layer 0 = stem, 1 = stage 0 transposed conv, 2 = stage 0 residual unit
    (preformed operand), 9 = stage 2 transposed conv, 10 = a stage 2 residual
    unit (per-layer launch: a four-stream step has fewer stage-2 tiles than
    SMs), 14 / 20 = residual units of stages 3 / 4, which run as the fused
    stage kernels (their first MMA waits for the gate; stage 4's writes stage
    5's planes)."""
    gate = torch.zeros(1, dtype=torch.int32, device="cuda")  # nothing ever sets it
    failing, clean = Run(lib, plan), Run(lib, plan)
    for _ in range(2):
        a, sa = failing.step()
        b, sb = clean.step()
        assert sa == sb == 0 and torch.equal(a, b)
    committed = failing.pool.clone()
    _, status = failing.step(gated_layer=layer, gate=gate)
    assert status in TIMEOUT_CODES, hex(status)
    assert failing.steps == 2
    # The step wrote only outside the committed windows and into the unread head table.
    assert torch.equal(committed_windows(failing.pool), committed_windows(committed))
    # The next ordinary steps continue from the committed history as if nothing had failed.
    for _ in range(2):
        a, sa = failing.step()
        b, sb = clean.step()
        assert sa == sb == 0
        assert torch.isfinite(a).all()
        assert torch.equal(a, b)


def test_ordinary_step_after_timeouts_is_unchanged(lib, plan):
    """The CUDA context stays usable: a fresh run after the gated launches equals a fresh run before them."""
    first = Run(lib, plan)
    a, _ = first.step()
    gate = torch.zeros(1, dtype=torch.int32, device="cuda")
    _, status = Run(lib, plan).step(gated_layer=5, gate=gate)
    assert status in TIMEOUT_CODES
    b, sb = Run(lib, plan).step()
    assert sb == 0 and torch.equal(a, b)
