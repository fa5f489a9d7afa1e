"""The fused kernels against the per-layer kernels on a B200 (``-m gpu``).

A whole step runs stage 5's three residual units and the final conv as one
kernel, and the three residual units of stages 2, 3 and 4 (256, 128 and 64
channels) with the next transposed conv's planes as one kernel each; all of them keep
each 128-row tile and its halo in shared memory. The same step with every
layer as its own kernel (``fav_debug_step_unfused``) is the check: both
compute each row with the same depthwise, Snake and f16 projection
arithmetic, and differ only in the final conv's summation order, so audio
agrees to 1e-5 and every history window (what the next step reads) to 1e-5
over consecutive steps with carried state, fresh streams and stream ends at
every tile position of the stage. The stage 2-4 windows, which no summation
order touches, are equal bit for bit. The cases cover partial last tiles of
32, 64 and 96 rows, warm-up tiles (CTA ranges that start inside a stream) and
both launch shapes of the 64-channel kernel.
"""
import ctypes as ct

import numpy as np
import pytest
import torch

from fast_audiovae import _native, build
from fast_audiovae import weights as W
from oracle.decoder import Decoder, discrepancy

pytestmark = pytest.mark.gpu

AUDIO_TOL = 1e-5
STATE_TOL = 1e-5


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not build.LIBRARY.exists():
        build.build()
    lib = _native.load_library()
    assert lib.fav_device_supported(), "not an sm_100 GPU"
    return lib


@pytest.fixture(scope="module")
def weights0():
    return W.seeded_weights(0)


@pytest.fixture(scope="module")
def plan(lib, weights0):
    return _native.Plan(weights0)


def ptr(t):
    return ct.c_void_p(t.data_ptr())


def run_steps(lib, plan, entry, latents, chunk_frames):
    """Decode ``latents`` [S,64,T] as consecutive steps of ``chunk_frames``
    through ``entry``; returns (audio [S, 1920T], state pool after each step)."""
    S, _, T = latents.shape
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    pool = torch.zeros(lib.fav_state_pool_bytes(S) // 4, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    audio = []
    pools = []
    for i, t in enumerate(range(0, T, chunk_frames)):
        f = min(chunk_frames, T - t)
        z = torch.from_numpy(np.ascontiguousarray(latents[:, :, t:t + f])).cuda()
        out = torch.empty(S, 1920 * f, device="cuda")
        ws_bytes = lib.fav_plan_workspace_bytes(plan.handle, S, f)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        # Head table parity alternates; the first step starts every stream fresh.
        codes = torch.tensor([(s << 2) | (2 if i == 0 else 0) | (i & 1) for s in range(S)], dtype=torch.int32,
                             device="cuda")
        _native.check(lib, entry(plan.handle, ptr(pool), S, ptr(codes), S, f, ptr(z), ptr(out), ptr(ws), ws_bytes,
                                 ptr(status), stream))
        torch.cuda.synchronize()
        assert status.item() == 0, hex(status.item())
        audio.append(out.cpu())
        pools.append(pool.cpu().clone())
    return torch.cat(audio, 1).numpy(), pools


# Float offsets of the stage 2-4 residual rings inside a slot, and their end
# (the stage-5 transposed conv's history ring follows): each history of H rows
# x C channels owns 2H ring rows at twice its reference state offset.
def _stage_rings():
    off = 6 * 64
    spans = []
    for i in range(6):
        cin = 2048 >> i
        off += cin
        for d in (1, 3, 9):
            if i in (2, 3, 4):
                spans.append((2 * off, 2 * (off + 6 * d * cin // 2)))
            off += 6 * d * cin // 2
    return spans


@pytest.mark.parametrize("streams,frames,chunk", [(1, 1, 1), (3, 5, 2), (2, 6, 3), (24, 2, 1), (64, 3, 3)])
def test_fused_tail_matches_per_layer_kernels(lib, plan, streams, frames, chunk):
    lat = np.concatenate([W.seeded_latents(400 + s, frames) for s in range(streams)], 0)
    fused, fused_pools = run_steps(lib, plan, lib.fav_step, lat, chunk)
    unfused, unfused_pools = run_steps(lib, plan, lib.fav_debug_step_unfused, lat, chunk)
    assert np.abs(fused - unfused).max() <= AUDIO_TOL
    stride = lib.fav_state_pool_bytes(1) // 4
    for a, b in zip(fused_pools, unfused_pools):
        diff = (a - b).abs().view(streams, stride).amax(0)
        bad = torch.nonzero(diff > STATE_TOL).flatten()
        assert bad.numel() == 0, f"slot floats {bad[:4].tolist()}..{bad[-1:].tolist()} differ by {float(diff.max())}"
        for lo, hi in _stage_rings():
            sa = a.view(streams, stride)[:, lo:hi]
            sb = b.view(streams, stride)[:, lo:hi]
            assert torch.equal(sa, sb), (lo, hi)


def test_fused_step_matches_oracle(lib, plan, weights0):
    """Three streams, four one-frame steps through the fused path, against the fp32 oracle."""
    lat = np.concatenate([W.seeded_latents(500 + s, 4) for s in range(3)], 0)
    got, _ = run_steps(lib, plan, lib.fav_step, lat, 1)
    oracle = Decoder(weights0)
    for s in range(3):
        want = oracle.decode_numpy(lat[s:s + 1])[0, 0]
        d = discrepancy(want, got[s])
        assert d["max_abs"] <= 2e-3 and d["snr_db"] >= 45.0, d
