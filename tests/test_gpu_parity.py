"""CUDA decoder parity on a B200 (``-m gpu``), through the C ABI and the facade.

Tolerances (the path's stated gates): against the reference fp32 output,
max-abs error <= 2e-3 and SNR >= 45 dB; streaming output concatenated chunk by
chunk is bit-identical to the same GPU's batch output. Engine and layer checks
use tighter, operand-precision-derived bounds given in each test.
"""
import ctypes as ct

import numpy as np
import pytest
import torch

from fast_audiovae import _native, build
from fast_audiovae import weights as W
from oracle.decoder import Decoder, discrepancy

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3
SNR_DB = 45.0


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


@pytest.fixture(scope="module")
def oracle0(weights0):
    torch.set_num_threads(max(1, torch.get_num_threads()))
    return Decoder(weights0)


@pytest.fixture(scope="module")
def batch_dec(lib, weights0):
    from fast_audiovae.cuda import CUDADecoder
    return CUDADecoder(weights0, {}, "batch")


@pytest.fixture(scope="module")
def stream_dec(lib, weights0):
    from fast_audiovae.cuda import CUDADecoder
    return CUDADecoder(weights0, {}, "streaming", max_streams=300)


def ptr(t):
    return ct.c_void_p(t.data_ptr())


def stream_handle():
    return ct.c_void_p(torch.cuda.current_stream().cuda_stream)


def layer_output(lib, plan, zs, last_layer):
    """Run layers 0..last_layer (zero history); return (workspace, float offset of the output)."""
    S, T = len(zs), zs[0].shape[2]
    z = torch.from_numpy(np.concatenate(zs, 0)).cuda()
    ws_bytes = lib.fav_step_workspace_bytes(S, T)
    ws = torch.empty(ws_bytes // 4, dtype=torch.float32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ct.c_void_p()
    _native.check(lib, lib.fav_debug_step_layers(plan.handle, None, 0, None, S, T, ptr(z), ptr(ws), ws_bytes,
                                                 ptr(status), last_layer, ct.byref(out), stream_handle()))
    torch.cuda.synchronize()
    assert status.item() == 0
    return ws, (out.value - ws.data_ptr()) // 4


def run_gemm(lib, m, n, k, mode, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g)
    b = torch.randn(n, k, generator=g)
    a_dev = a.cuda()
    c = torch.full((m, n), float("nan"), device="cuda")
    _native.check(lib, lib.fav_test_gemm(ptr(a_dev), m, k, b.numpy().ctypes.data_as(ct.c_void_p), n, mode, ptr(c),
                                         stream_handle()))
    return a, b, c.cpu()


@pytest.mark.parametrize("m,n,k", [(1, 32, 64), (128, 256, 64), (200, 64, 128), (300, 512, 256), (128, 128, 32),
                                   (129, 256, 1024), (640, 128, 2048)])
def test_engine_f16(lib, m, n, k):
    """f16 operands, fp32 accumulate: equals the fp64 product of f16-rounded operands to ~1e-6."""
    a, b, c = run_gemm(lib, m, n, k, 0, m + n + k)
    ref = a.half().double() @ b.half().double().T
    assert (c.double() - ref).abs().max() <= 1e-5 * ref.abs().max() + 1e-6


@pytest.mark.parametrize("m,n,k", [(1, 32, 64), (128, 256, 64), (300, 512, 256), (129, 256, 1024), (77, 64, 4096)])
def test_engine_split_bf16(lib, m, n, k):
    """Split-bf16 (three MMAs): within ~2^-16 of the exact fp32 product."""
    a, b, c = run_gemm(lib, m, n, k, 1, 3 * m + n + k)
    ref = a.double() @ b.double().T
    assert (c.double() - ref).abs().max() <= 3e-5 * ref.abs().max()


@pytest.mark.parametrize("streams,frames", [(2, 3), (5, 1), (1, 7)])
def test_every_layer_matches_oracle(lib, plan, oracle0, streams, frames):
    """Each of the 25 projection layers (zero history) against the oracle's layer output."""
    zs = [W.seeded_latents(100 + s, frames) for s in range(streams)]
    traces = []
    for z in zs:
        trace = []
        oracle0.decode(z, trace=trace)
        traces.append(trace)
    for layer in range(25):
        ws, off = layer_output(lib, plan, zs, layer)
        ref = torch.cat([t[layer][0].T for t in traces], 0)
        got = ws[off:off + ref.numel()].view(ref.shape).cpu()
        rel = (got.double() - ref.double()).norm() / ref.double().norm()
        assert rel < 5e-4, (layer, float(rel))


def test_batch_matches_reference_fp32_output(golden, batch_dec):
    """cfg1: latents [1,64,25] seed 0 against the reference decoder's own output."""
    g = golden("decoder_seed0.npz")
    for key in ("3", "25"):
        d = discrepancy(g["audio" + key], batch_dec.decode(g["z" + key]))
        assert d["max_abs"] <= MAX_ABS and d["snr_db"] >= SNR_DB, d


@pytest.mark.parametrize("seed,frames", [(1, 25), (2, 40), (3, 1), (4, 2)])
def test_batch_matches_oracle(batch_dec, oracle0, seed, frames):
    z = W.seeded_latents(seed, frames)
    d = discrepancy(oracle0.decode_numpy(z), batch_dec.decode(z))
    assert d["max_abs"] <= MAX_ABS and d["snr_db"] >= SNR_DB, d


def test_other_weights_seed(lib):
    from fast_audiovae.cuda import CUDADecoder
    w = W.seeded_weights(7)
    dec = CUDADecoder(w, {}, "batch")
    z = W.seeded_latents(7, 25)
    d = discrepancy(Decoder(w).decode_numpy(z), dec.decode(z))
    assert d["max_abs"] <= MAX_ABS and d["snr_db"] >= SNR_DB, d


def decode_pattern(stream, z, pattern):
    parts, start, k = [], 0, 0
    while start < z.shape[2]:
        end = min(z.shape[2], start + pattern[k % len(pattern)])
        parts.append(stream.decode_chunk(z[..., start:end]))
        start, k = end, k + 1
    assert stream.flush().shape == (1, 1, 0)
    return np.concatenate(parts, -1)


def test_cfg2_stream_of_250_frames_is_bitwise_batch(batch_dec, stream_dec):
    """cfg2: 250 one-frame chunks + flush == batch decode of [1,64,250], bit for bit."""
    z = W.seeded_latents(0, 250)
    full = batch_dec.decode(z)
    with stream_dec.stream() as s:
        streamed = decode_pattern(s, z, (1,))
    assert np.array_equal(full.view(np.uint32), streamed.view(np.uint32))


@pytest.mark.parametrize("pattern", [(1,), (2,), (5,), (1, 7, 2, 3, 11)])
def test_streaming_patterns_bitwise(batch_dec, stream_dec, pattern):
    """``tools/validate_streaming.py:145-149`` patterns, gated bit-exact here."""
    z = W.seeded_latents(11, 31)
    full = batch_dec.decode(z)
    with stream_dec.stream() as s:
        assert np.array_equal(decode_pattern(s, z, pattern), full)


def test_final_partial_reset_and_interleaving(batch_dec, stream_dec):
    """``tools/validate_streaming.py:156-191``: final partial chunk, reset, interleaved streams."""
    z = W.seeded_latents(12, 23)
    full = batch_dec.decode(z)
    partial = z[..., :7]
    with stream_dec.stream() as s:
        assert np.array_equal(decode_pattern(s, partial, (6,)), batch_dec.decode(partial))
    with stream_dec.stream() as s:
        s.decode_chunk(z[..., :1])
        s.reset()
        assert np.array_equal(decode_pattern(s, z, (5,)), full)
        s.reset()
        assert np.array_equal(decode_pattern(s, z, (5,)), full)
    other = np.ascontiguousarray(z[..., ::-1])
    other_full = batch_dec.decode(other)
    with stream_dec.stream() as a, stream_dec.stream() as b:
        outs = [[], []]
        start, k = 0, 0
        while start < 23:
            end = min(23, start + (2, 5, 1)[k % 3])
            outs[0].append(a.decode_chunk(z[..., start:end]))
            outs[1].append(b.decode_chunk(other[..., start:end]))
            start, k = end, k + 1
    assert np.array_equal(np.concatenate(outs[0], -1), full)
    assert np.array_equal(np.concatenate(outs[1], -1), other_full)


def test_many_streams_per_step_bitwise(batch_dec, stream_dec):
    """cfg3 shape: 256 streams x 2-frame chunks in one step per chunk; each equals its batch decode."""
    n, steps = 256, 3
    zs = [W.seeded_latents(1000 + i, 2 * steps) for i in range(n)]
    streams = [stream_dec.stream() for _ in range(n)]
    got = [[] for _ in range(n)]
    for t in range(steps):
        for i, audio in enumerate(stream_dec.decode_streams(streams, [z[..., 2 * t:2 * t + 2] for z in zs])):
            got[i].append(audio)
    for s in streams:
        s.close()
    refs = batch_dec.decode_many(zs)
    for i in range(n):
        assert np.array_equal(np.concatenate(got[i], -1), refs[i]), i


def test_step_into_mapped_host_memory(lib, plan, stream_dec):
    """fav_step writing its audio through a pinned buffer's mapped address
    equals the same step into device memory, bit for bit; pageable memory has
    no device address; the streaming facade takes the mapped path."""
    S, F = 5, 2
    pinned = torch.empty(S * 1920 * F, dtype=torch.float32, pin_memory=True)
    dev_ptr = ct.c_void_p()
    assert lib.fav_host_device_pointer(ct.c_void_p(pinned.data_ptr()), ct.byref(dev_ptr)) == 0
    pageable = np.zeros(64, np.float32)
    assert lib.fav_host_device_pointer(ct.c_void_p(pageable.ctypes.data), ct.byref(ct.c_void_p())) != 0
    lat = torch.from_numpy(np.concatenate([W.seeded_latents(70 + s, F) for s in range(S)], 0)).cuda()
    ws_bytes = lib.fav_plan_workspace_bytes(plan.handle, S, F)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    codes = torch.tensor([(s << 2) | 2 for s in range(S)], dtype=torch.int32, device="cuda")
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    outs = []
    for target in (None, dev_ptr):
        pool = torch.zeros(lib.fav_state_pool_bytes(S) // 4, device="cuda")
        dev_audio = torch.empty(S, 1920 * F, device="cuda")
        audio = target if target is not None else ct.c_void_p(dev_audio.data_ptr())
        _native.check(lib, lib.fav_step(plan.handle, ct.c_void_p(pool.data_ptr()), S, ct.c_void_p(codes.data_ptr()),
                                        S, F, ct.c_void_p(lat.data_ptr()), audio, ct.c_void_p(ws.data_ptr()),
                                        ws_bytes, ct.c_void_p(status.data_ptr()), stream))
        torch.cuda.synchronize()
        assert status.item() == 0
        outs.append(dev_audio.cpu().numpy() if target is None else pinned.numpy().reshape(S, -1).copy())
    assert np.array_equal(outs[0], outs[1])
    with stream_dec.stream() as s:
        s.decode_chunk(W.seeded_latents(3, 1))
    assert any(v is not None for v in stream_dec._backend.mapped.values())


def test_decode_many_equals_single_decodes(batch_dec):
    zs = [W.seeded_latents(40 + i, 9) for i in range(5)]
    many = batch_dec.decode_many(zs)
    for z, audio in zip(zs, many):
        assert np.array_equal(audio, batch_dec.decode(z))


def test_histories_hold_reference_values(lib, plan, oracle0):
    """After one step the slot's history windows hold the reference's 26 histories.

    Pool layout: per slot, rings of 2H rows (channels last) for each history at
    twice its reference offset, then two head tables of 32 int32; a step from
    read table 0 writes its heads to table 1. A transposed conv's one-row
    history holds its activated input as the split-bf16 pair the MMA consumes,
    packed per channel as (hi << 16) | lo; hi + lo is the fp32 value to 2^-16
    relative.
    """
    z = W.seeded_latents(21, 3)
    pool = torch.zeros(lib.fav_state_pool_bytes(2) // 4, device="cuda")
    codes = torch.tensor([(1 << 2) | 2 | 0], dtype=torch.int32, device="cuda")  # slot 1, fresh, read table 0
    zd = torch.from_numpy(z).cuda()
    audio = torch.empty(1920 * 3, device="cuda")
    ws_bytes = lib.fav_step_workspace_bytes(1, 3)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    _native.check(lib, lib.fav_step(plan.handle, ptr(pool), 2, ptr(codes), 1, 3, ptr(zd), ptr(audio), ptr(ws),
                                    ws_bytes, ptr(status), stream_handle()))
    torch.cuda.synchronize()
    assert status.item() == 0
    _, states = oracle0.decode(z)
    slots = pool.view(2, _native.SLOT_STRIDE_FLOATS)
    assert not slots[0].any()
    slot = slots[1].cpu()
    heads = slot[2 * _native.SLOT_FLOATS:].view(torch.int32)[32:64].numpy()
    rings = slot[:2 * _native.SLOT_FLOATS].numpy()
    off = 0
    for index, (name, shape) in enumerate(W.state_shapes().items()):
        _, channels, rows = shape
        ring = rings[2 * off:2 * off + 2 * rows * channels].reshape(2 * rows, channels)
        window = ring[(heads[index] + np.arange(rows)) % (2 * rows)]
        if name.endswith("transpose.history"):
            bits = window.view(np.uint32)
            window = (bits & 0xFFFF0000).view(np.float32) + (bits << 16).view(np.float32)
        got = window.T[None]
        ref = states[name].numpy()
        scale = max(1.0, float(np.abs(ref).max()))
        assert np.abs(got - ref).max() <= 2e-3 * scale, name
        off += rows * channels
    assert off == _native.SLOT_FLOATS


def test_repeat_is_deterministic(batch_dec):
    z = W.seeded_latents(5, 13)
    a = batch_dec.decode(z)
    b = batch_dec.decode(z)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_long_clip_chunking_is_bitwise(lib, weights0, oracle0):
    """cfg4's clip length (750 frames, 30 s): chunk sizes 128 and 50 give
    identical bits, and the whole clip meets the fp32 gates against the oracle."""
    from fast_audiovae.cuda import CUDADecoder
    z = W.seeded_latents(63, 750)
    a = CUDADecoder(weights0, {}, "batch", batch_chunk_frames=128).decode(z)
    b = CUDADecoder(weights0, {}, "batch", batch_chunk_frames=50).decode(z)
    assert np.array_equal(a, b)
    d = discrepancy(oracle0.decode_numpy(z), a)
    assert d["max_abs"] <= MAX_ABS and d["snr_db"] >= SNR_DB, d


def test_benchmarked_step_matches_oracle(lib, plan, oracle0):
    """The benchmark's own step: 512 streams x 1-frame chunks (seed = stream id)
    through fav_step, three carried steps; eight of the streams (first and
    last slot among them) against the oracle's decode of the same three frames."""
    S, steps = 512, 3
    lat = np.stack([W.seeded_latents(s, steps)[0] for s in range(S)])  # [S, 64, steps]
    pool = torch.zeros(lib.fav_state_pool_bytes(S) // 4, device="cuda")
    ws_bytes = lib.fav_plan_workspace_bytes(plan.handle, S, 1)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    audio = torch.empty(steps, S, 1920, device="cuda")
    for t in range(steps):
        codes = torch.tensor([(s << 2) | (2 if t == 0 else 0) | (t & 1) for s in range(S)], dtype=torch.int32,
                             device="cuda")
        z = torch.from_numpy(np.ascontiguousarray(lat[:, :, t:t + 1])).cuda()
        _native.check(lib, lib.fav_step(plan.handle, ptr(pool), S, ptr(codes), S, 1, ptr(z), ptr(audio[t]), ptr(ws),
                                        ws_bytes, ptr(status), stream_handle()))
    torch.cuda.synchronize()
    assert status.item() == 0
    got = audio.permute(1, 0, 2).reshape(S, 1, 1, steps * 1920).cpu().numpy()
    for s in (0, 1, 63, 64, 255, 256, 510, 511):
        d = discrepancy(oracle0.decode_numpy(lat[s:s + 1]), got[s])
        assert d["max_abs"] <= MAX_ABS and d["snr_db"] >= SNR_DB, (s, d)


def test_cfg3_full_run_is_bitwise_batch(lib, weights0, stream_dec):
    """cfg3 in full: 256 streams x 2-frame chunks for 125 steps (10 s per
    stream), one step per chunk for all streams; every stream equals its batch
    decode bit for bit."""
    from fast_audiovae.cuda import CUDADecoder
    n, steps, F = 256, 125, 2
    zs = [W.seeded_latents(s, F * steps) for s in range(n)]
    streams = [stream_dec.stream() for _ in range(n)]
    got = np.empty((n, 1920 * F * steps), np.float32)
    for t in range(steps):
        for i, audio in enumerate(stream_dec.decode_streams(streams, [z[..., F * t:F * (t + 1)] for z in zs])):
            got[i, 1920 * F * t:1920 * F * (t + 1)] = audio[0, 0]
    for s in streams:
        s.close()
    batch = CUDADecoder(weights0, {}, "batch", batch_chunk_frames=25)
    for g in range(0, n, 64):
        for i, ref in enumerate(batch.decode_many(zs[g:g + 64])):
            assert np.array_equal(got[g + i].view(np.uint32), ref[0, 0].view(np.uint32)), g + i


def test_public_load_api(lib):
    import fast_audiovae
    dec = fast_audiovae.load(mode="batch", device="cuda")
    assert dec.info["device"] == "cuda" and dec.info["sm_count"] > 0
    z = W.seeded_latents(0, 2)
    assert dec.decode(z).shape == (1, 1, 3840)
    sdec = fast_audiovae.load(mode="stream", device="cuda", max_streams=4)
    with sdec.stream() as s:
        assert s.decode_chunk(z).shape == (1, 1, 3840)
        assert s.frames_decoded == 2
