"""Facade contract of the CUDA route with a fake backend (CPU, no GPU, no torch.cuda).

Restates the reference's facade tests (``tests/test_gpu_api.py``,
``tests/test_streaming_runtime.py``) for ``fast_audiovae.cuda``: validation
before device work, mode misuse, empty chunks, reset/flush/close, transactional
history (a failed step never advances a stream), independent interleaved
streams and serialised device access. The fake backend keeps the double-buffered
history pool of the C ABI (read one half, write the other) and computes with
the oracle.
"""
import threading
import time

import numpy as np
import pytest
import torch

from fast_audiovae import cuda as C
from fast_audiovae import weights as W
from oracle.decoder import Decoder


class FakeBackend:
    def __init__(self, weights):
        self.oracle = Decoder(weights)
        self.pool = {}
        self.calls = 0
        self.fail_next = False
        self.active = 0
        self.max_active = 0
        self.plan_bytes = 123

    def step(self, codes, arrays, frames):
        self.active += 1
        self.max_active = max(self.max_active, self.active)
        try:
            self.calls += 1
            time.sleep(0.001)
            out = []
            for code, z in zip(codes, arrays):
                z = z if z.ndim == 3 else z[None]  # a stacked [n, 64, L] step yields [64, L] rows
                slot, fresh, half = code >> 2, bool(code & 2), code & 1
                states = None if fresh else self.pool.get((slot, half))
                audio, new = self.oracle.decode(z, states)
                self.pool[(slot, half ^ 1)] = new  # written before any failure, like the device
                out.append(audio.numpy().reshape(-1))
            if self.fail_next:
                self.fail_next = False
                raise RuntimeError("injected device failure")
            return np.stack(out).astype(np.float32)
        finally:
            self.active -= 1

    def decode_many(self, arrays, frames):
        self.calls += 1
        return np.stack([self.oracle.decode_numpy(z).reshape(-1) for z in arrays]).astype(np.float32)


@pytest.fixture(scope="module")
def weights():
    return W.seeded_weights(0)


def make(weights, mode="streaming", **kw):
    backend = FakeBackend(weights)
    return C.CUDADecoder(weights, {"device": "cuda"}, mode, backend=backend, **kw), backend


def test_mode_misuse_and_info(weights):
    dec, _ = make(weights, "batch")
    with pytest.raises(RuntimeError, match="stream"):
        dec.stream()
    sdec, _ = make(weights, "streaming")
    with pytest.raises(RuntimeError, match="stream"):
        sdec.decode(W.seeded_latents(0, 1))
    assert sdec.info["state_bytes_per_stream"] == 647424 and sdec.info["output_device"] == "cpu"


@pytest.mark.parametrize("bad", [
    np.zeros((1, 64, 2), np.float64), np.zeros((64, 2), np.float32), np.zeros((1, 63, 2), np.float32),
    np.full((1, 64, 2), np.nan, np.float32), [[0.0]], np.full((1, 64, 1), np.inf, np.float32)])
def test_validation_precedes_device_work(weights, bad):
    dec, backend = make(weights, "batch")
    with pytest.raises(ValueError):
        dec.decode(bad)
    sdec, sbackend = make(weights)
    with sdec.stream() as s, pytest.raises(ValueError):
        s.decode_chunk(bad)
    assert backend.calls == sbackend.calls == 0


def test_empty_inputs(weights):
    dec, backend = make(weights, "batch")
    assert dec.decode(np.zeros((1, 64, 0), np.float32)).shape == (1, 1, 0)
    sdec, sbackend = make(weights)
    with sdec.stream() as s:
        assert s.decode_chunk(np.zeros((1, 64, 0), np.float32)).shape == (1, 1, 0)
        assert s.flush().shape == (1, 1, 0) and s.frames_decoded == 0
    assert backend.calls == sbackend.calls == 0


def test_batch_output_is_owned_fp32(weights):
    dec, _ = make(weights, "batch")
    z = W.seeded_latents(1, 2)
    before = z.copy()
    audio = dec.decode(z)
    assert audio.dtype == np.float32 and audio.shape == (1, 1, 3840)
    assert np.array_equal(z, before)
    np.testing.assert_array_equal(audio, Decoder(weights).decode_numpy(z))


def test_chunked_stream_equals_batch_and_reset(weights):
    sdec, _ = make(weights)
    z = W.seeded_latents(2, 5)
    full = Decoder(weights).decode_numpy(z)
    with sdec.stream() as s:
        parts = [s.decode_chunk(z[..., a:b]) for a, b in ((0, 1), (1, 3), (3, 5))]
        assert s.frames_decoded == 5
        np.testing.assert_allclose(np.concatenate(parts, -1), full, atol=1e-5)
        s.reset()
        assert s.frames_decoded == 0
        again = np.concatenate([s.decode_chunk(z[..., :2]), s.decode_chunk(z[..., 2:])], -1)
        np.testing.assert_allclose(again, full, atol=1e-5)


def test_failed_step_does_not_advance_history(weights):
    sdec, backend = make(weights)
    z = W.seeded_latents(3, 4)
    full = Decoder(weights).decode_numpy(z)
    with sdec.stream() as s:
        first = s.decode_chunk(z[..., :2])
        backend.fail_next = True
        with pytest.raises(RuntimeError, match="injected"):
            s.decode_chunk(W.seeded_latents(99, 2))
        assert s.frames_decoded == 2
        second = s.decode_chunk(z[..., 2:])
    np.testing.assert_allclose(np.concatenate([first, second], -1), full, atol=1e-5)


def test_closed_stream_and_slot_reuse(weights):
    sdec, _ = make(weights, max_streams=2)
    a, b = sdec.stream(), sdec.stream()
    with pytest.raises(RuntimeError, match="slots"):
        sdec.stream()
    a.close()
    a.close()
    with pytest.raises(RuntimeError, match="closed"):
        a.decode_chunk(W.seeded_latents(0, 1))
    with pytest.raises(RuntimeError, match="closed"):
        a.reset()
    c = sdec.stream()
    assert c._fresh
    b.close()
    c.close()


def test_interleaved_streams_are_independent(weights):
    sdec, _ = make(weights)
    za, zb = W.seeded_latents(4, 5), W.seeded_latents(5, 5)
    oracle = Decoder(weights)
    with sdec.stream() as a, sdec.stream() as b:
        outs = [[], []]
        for lo, hi in ((0, 2), (2, 4), (4, 5)):
            outs[0].append(a.decode_chunk(za[..., lo:hi]))
            outs[1].append(b.decode_chunk(zb[..., lo:hi]))
    np.testing.assert_allclose(np.concatenate(outs[0], -1), oracle.decode_numpy(za), atol=1e-5)
    np.testing.assert_allclose(np.concatenate(outs[1], -1), oracle.decode_numpy(zb), atol=1e-5)


def test_decode_streams_batches_and_commits_together(weights):
    sdec, backend = make(weights)
    zs = [W.seeded_latents(10 + i, 4) for i in range(3)]
    oracle = Decoder(weights)
    streams = [sdec.stream() for _ in zs]
    got = [[] for _ in zs]
    for lo in (0, 2):
        for i, audio in enumerate(sdec.decode_streams(streams, [z[..., lo:lo + 2] for z in zs])):
            got[i].append(audio)
    assert backend.calls == 2
    for z, parts in zip(zs, got):
        np.testing.assert_allclose(np.concatenate(parts, -1), oracle.decode_numpy(z), atol=1e-5)
    backend.fail_next = True
    with pytest.raises(RuntimeError):
        sdec.decode_streams(streams, [W.seeded_latents(0, 1)] * 3)
    assert all(s.frames_decoded == 4 for s in streams)
    with pytest.raises(ValueError, match="once"):
        sdec.decode_streams([streams[0], streams[0]], [zs[0][..., :1]] * 2)
    with pytest.raises(ValueError, match="equal"):
        sdec.decode_streams(streams[:2], [zs[0][..., :1], zs[1][..., :2]])


def test_device_work_is_serialised(weights):
    sdec, backend = make(weights)
    z = W.seeded_latents(6, 1)
    streams = [sdec.stream() for _ in range(4)]
    threads = [threading.Thread(target=lambda s=s: [s.decode_chunk(z) for _ in range(3)]) for s in streams]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert backend.max_active == 1 and backend.calls == 12


def test_load_rejects_other_devices_and_threads():
    import fast_audiovae
    with pytest.raises(ValueError, match="cuda"):
        fast_audiovae.load(device="cpu")
    with pytest.raises(ValueError, match="threads"):
        fast_audiovae.load(threads=2)
    with pytest.raises(ValueError, match="mode"):
        fast_audiovae.load(mode="both")
    info = fast_audiovae.setup(mode="stream")
    assert info["mode"] == "streaming" and info["fallback"] is False


def test_load_without_gpu_never_falls_back():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import fast_audiovae
    with pytest.raises(RuntimeError, match="CUDA"):
        fast_audiovae.load(mode="batch")


def test_lent_output_buffers_are_reused_only_after_release():
    """Returned audio lives in a pooled host buffer until its last view is gone."""
    import gc

    import torch

    from fast_audiovae.cuda import LentBuffers

    made = []

    def alloc(numel):
        made.append(torch.zeros(numel))
        return made[-1]

    pool = LentBuffers(alloc, limit=2)
    a = pool.lend(buf := pool.acquire(8), buf[:8].numpy())
    views = list(a.reshape(2, 1, 1, 4))
    del a, buf
    gc.collect()
    assert pool.lent == 1  # the views keep the buffer lent
    b_buf = pool.acquire(8)
    assert len(made) == 2 and b_buf is made[1]
    assert pool.acquire(8) is None  # limit reached: caller copies instead
    del views
    gc.collect()
    assert pool.lent == 1
    assert pool.acquire(8) is made[0]  # released buffer comes back
