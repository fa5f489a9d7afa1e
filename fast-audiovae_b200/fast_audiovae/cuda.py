"""Explicit CUDA (B200, sm_100a) decoding: the drop-in for the reference GPU route.

Mirrors ``src/fast_audiovae/gpu.py`` of bevenky/fast-audiovae:

* ``CUDADecoder`` <- ``GPUDecoder`` (``gpu.py:125-199``): immutable device weights
  shared by independent streams, one lock serialising device work, input
  validation before any device work (``gpu.py:115-122``), owned CPU-ready fp32
  output, finite check before commit (``gpu.py:177-179``), mode misuse raises
  ``RuntimeError`` (``gpu.py:189-198``).
* ``CUDAStream`` <- ``GPUStream`` (``gpu.py:202-249``): per-stream history that
  advances only after a successful step (``gpu.py:216-225``), ``reset``,
  ``flush`` (always ``[1,1,0]``), ``close`` and context management.

Device work runs in ``libfav_cuda.so`` through its C ABI (``DeviceBackend``);
torch only supplies device memory, pinned host buffers and the CUDA stream.
There is no CPU path: an explicit CUDA request never falls back
(``gpu.py:29-41``). As the reference injects its model and torch module into
``GPUDecoder``, the backend is a constructor argument, which lets the facade
contract be tested without a GPU.

Beyond the reference, ``CUDADecoder.decode_streams`` decodes one chunk for
many streams in a single step (one kernel launch per layer for all of them),
and ``decode_many`` batch-decodes several equal-length clips at once.
"""
from __future__ import annotations

import collections
import ctypes as ct
import threading
import weakref
from operator import attrgetter

import numpy as np

from . import weights as W

HOP = W.HOP_SAMPLES
STATE_BYTES = W.STATE_BYTES_FP32
_FRESH = 2

# Per-stream fields read with ``map`` so a step over hundreds of streams loops in C.
_DTYPE, _SHAPE = attrgetter("dtype"), attrgetter("shape")
_DECODER, _LOCK, _CLOSED = attrgetter("_decoder"), attrgetter("_lock"), attrgetter("_closed")
_SLOT = attrgetter("_slot")
_LOCK_ACQUIRE, _LOCK_RELEASE = type(threading.Lock()).acquire, type(threading.Lock()).release


def _drain(iterator):
    collections.deque(iterator, maxlen=0)


def _latents(value):
    """``gpu.py:115-122``: float32 numpy ``[1,64,L]``, finite; owned C-contiguous copy."""
    if (not isinstance(value, np.ndarray) or value.dtype != np.float32
            or value.ndim != 3 or value.shape[:2] != (1, 64)):
        raise ValueError("Latents must be a float32 NumPy array with shape [1,64,L]")
    if not np.isfinite(value).all():
        raise ValueError("Latents must contain only finite values")
    return np.array(value, copy=True, order="C") if value.shape[2] else value


def _latents_step(chunks, stage=None):
    """``gpu.py:115-122`` for one step of many streams: every chunk a float32
    ``[1,64,L]`` array of one common L, all finite. Returns the chunks stacked
    as an owned ``[n,64,L]`` array (one copy, one vectorised finiteness check),
    written into ``stage(n, L)`` (a backend's staging buffer) when given."""
    if not chunks:
        return np.empty((0, 64, 0), dtype=np.float32)
    # One pass each over types, dtypes and first dimensions (a server step
    # carries hundreds of chunks); concatenation then checks the other
    # dimensions. The per-chunk loop below only names a failure.
    first = chunks[0]
    if (set(map(type, chunks)) == {np.ndarray} and set(map(_DTYPE, chunks)) == {np.dtype(np.float32)}
            and set(map(len, chunks)) == {1} and first.ndim == 3 and first.shape[1] == 64):
        n, frames = len(chunks), first.shape[2]
        out = stage(n, frames) if stage is not None else None
        try:
            stacked = np.concatenate(chunks, axis=0, out=out)
        except ValueError:
            stacked = None
        if stacked is None or stacked.shape != (n, 64, frames):
            if any(c.ndim != 3 or c.shape[1] != 64 for c in chunks):
                raise ValueError("Latents must be a float32 NumPy array with shape [1,64,L]")
            raise ValueError("decode_streams requires chunks of equal length")
    else:
        for value in chunks:
            if (not isinstance(value, np.ndarray) or value.dtype != np.float32
                    or value.ndim != 3 or value.shape[:2] != (1, 64)):
                raise ValueError("Latents must be a float32 NumPy array with shape [1,64,L]")
        raise ValueError("decode_streams requires chunks of equal length")
    if not np.isfinite(stacked).all():
        raise ValueError("Latents must contain only finite values")
    return stacked


# Kernel status of a step whose audio was not finite (the final kernel's check).
NONFINITE_STATUS = 0x106


def _torch():
    try:
        import torch
    except ImportError as error:  # pragma: no cover - torch is a hard dependency here
        raise RuntimeError("CUDA decoding requires PyTorch for device buffers") from error
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is unavailable; an explicit CUDA request never falls back to CPU")
    return torch


class LentBuffers:
    """Host output buffers lent to returned audio arrays.

    A step's audio lands in a pinned buffer (written there by the kernels
    through its mapped device address, or copied from the device), and the
    caller receives NumPy arrays over that buffer; the buffer returns
    to the pool only when the last of those arrays is gone (a weakref
    finalizer), so no live result is ever overwritten. While more than
    ``limit`` results are held, ``acquire`` returns None and the caller copies
    into an ordinary owned array instead, so keeping results never pins more
    than ``limit`` buffers. ``alloc(numel)`` makes a buffer (a pinned fp32
    tensor in DeviceBackend).
    """

    def __init__(self, alloc, limit=4):
        self._alloc = alloc
        self._limit = limit
        self._free = []
        self._lent = 0
        self._lock = threading.Lock()

    def acquire(self, numel):
        with self._lock:
            for i, buf in enumerate(self._free):
                if buf.numel() >= numel:
                    self._lent += 1
                    return self._free.pop(i)
            if self._lent >= self._limit:
                return None
            self._lent += 1
        return self._alloc(numel)

    def release(self, buf):
        with self._lock:
            self._lent -= 1
            self._free.append(buf)

    def lend(self, buf, array):
        """Return ``buf`` to the pool once ``array`` and every view of it are gone."""
        weakref.finalize(array, self.release, buf)
        return array

    @property
    def lent(self):
        return self._lent


class DeviceBackend:
    """Device memory and C-ABI calls for one decoder (one plan, one history pool).

    ``step(codes, arrays, frames)`` and ``decode_many(arrays, frames)`` return
    fp32 audio ``[n, 1920*frames]`` after a synchronising download, raising
    ``RuntimeError`` on any launch, kernel-status or finiteness failure. A
    failed step may have written the *unread* half of a history slot only.
    """

    def __init__(self, weights, *, max_streams, device=0, batch_chunk_frames=128, precision=0, graphs=True):
        torch = _torch()
        from ._native import Plan, load_library
        self.torch = torch
        self.device = torch.device("cuda", device)
        self.max_streams = max_streams
        self.chunk = batch_chunk_frames
        with torch.cuda.device(self.device):
            self.lib = load_library()
            if not self.lib.fav_device_supported():
                raise RuntimeError("CUDA decoding requires an sm_100 (B200) GPU; no fallback is permitted")
            self.plan = Plan(weights, precision)
            self.pool = torch.zeros(self.lib.fav_state_pool_bytes(max_streams) // 4, dtype=torch.float32,
                                    device=self.device)
            self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
            self.status_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.cache = {}
        self.out_buffers = LentBuffers(lambda numel: torch.empty(numel, dtype=torch.float32, pin_memory=True))
        self.mapped = {}  # lent buffer host address -> its device address (None: not mapped)
        # Streaming steps replay a CUDA graph of the step's kernel launches per
        # (streams, frames, buffers): the first step of a shape runs eagerly,
        # the second captures, later ones replay (one launch call per step).
        self.graphs_enabled = graphs
        self.graphs = {}
        self.graph_seen = set()
        # (streams, frames, lent buffer) -> (staging view, graph, status view):
        # replayed without rebuilding the step's arguments.
        self.fast = {}

    @property
    def plan_bytes(self):
        return self.plan.device_bytes

    def _buffer(self, key, shape, dtype, pinned=False):
        t = self.cache.get(key)
        numel = int(np.prod(shape))
        if t is None or t.numel() < numel:
            torch = self.torch
            t = (torch.empty(numel, dtype=dtype, pin_memory=True) if pinned
                 else torch.empty(numel, dtype=dtype, device=self.device))
            self.cache[key] = t
            self.fast = {}  # replay entries point into the buffers they were captured with
        return t[:numel].view(*shape)

    @staticmethod
    def _ptr(tensor):
        return ct.c_void_p(tensor.data_ptr())

    def _stream(self):
        return ct.c_void_p(self.torch.cuda.current_stream(self.device).cuda_stream)

    def stage(self, n, frames):
        """Pinned host staging of one streaming step: latents ``[n, 64, frames]``
        fp32, then the slot codes and a zero status word, uploaded together by
        one copy. Returns the latents part as a writable NumPy view."""
        count = n * 64 * frames
        host = self._buffer("stage_host", (count + n + 1,), self.torch.float32, pinned=True)
        return host.numpy()[:count].reshape(n, 64, frames)

    def _upload(self, arrays, frames):
        n = len(arrays)
        host = self._buffer("z_host", (n, 64, frames), self.torch.float32, pinned=True)
        hn = host.numpy()
        if isinstance(arrays, np.ndarray):
            hn[...] = arrays  # already stacked [n, 64, frames]
        else:
            for i, a in enumerate(arrays):
                hn[i] = a[0]
        dev = self._buffer("z_dev", (n, 64, frames), self.torch.float32)
        dev.copy_(host, non_blocking=True)
        return dev

    def _mapped(self, buf):
        """Device address of pinned buffer ``buf``, or None when it is not mapped."""
        key = buf.data_ptr()
        if key not in self.mapped:
            dev = ct.c_void_p()
            ok = self.lib.fav_host_device_pointer(ct.c_void_p(key), ct.byref(dev)) == 0
            self.mapped[key] = dev.value if ok else None
        return self.mapped[key]

    def _finish(self, lent, status=None):
        """Synchronise and read the kernels' status; on failure the lent buffer
        goes back to the pool and the step raises."""
        self.status_host.copy_(self.status if status is None else status.view(self.torch.int32),
                               non_blocking=True)
        self.torch.cuda.current_stream(self.device).synchronize()
        status = int(self.status_host.item())
        if status:
            if lent is not None:
                self.out_buffers.release(lent)
            if status == NONFINITE_STATUS:
                raise RuntimeError("CUDA model returned nonfinite audio")
            raise RuntimeError("CUDA decoder kernel reported status 0x%x" % status)

    def _download(self, audio_dev, status=None):
        """The step's audio as host fp32: in a lent pinned buffer (no host copy),
        or, while too many earlier results are still held, an owned copy."""
        shape = tuple(audio_dev.shape)
        lent = self.out_buffers.acquire(audio_dev.numel())
        host = (lent[:audio_dev.numel()].view(*shape) if lent is not None
                else self._buffer("a_host", shape, self.torch.float32, pinned=True))
        host.copy_(audio_dev, non_blocking=True)
        self._finish(lent, status)
        if lent is None:
            return host.numpy().copy()
        return self.out_buffers.lend(lent, host.numpy())

    def _stage_latents(self, hn, arrays, n, count, frames):
        """Latents into the staging buffer (unless the caller stacked them there)."""
        if not (isinstance(arrays, np.ndarray) and arrays.ctypes.data == hn.ctypes.data):
            view = hn[:count].reshape(n, 64, frames)
            if isinstance(arrays, np.ndarray):
                view[...] = arrays
            else:
                for i, a in enumerate(arrays):
                    view[i] = a[0]

    def _check_status(self, status, lent):
        if status:
            if lent is not None:
                self.out_buffers.release(lent)
            if status == NONFINITE_STATUS:
                raise RuntimeError("CUDA model returned nonfinite audio")
            raise RuntimeError("CUDA decoder kernel reported status 0x%x" % status)

    def _replay(self, fast, lent, codes, arrays, n, frames):
        """A step whose graph (upload, kernels, status download) exists for
        these streams, frames and lent output buffer: stage, replay, read."""
        hn, graph, status_np = fast
        count = n * 64 * frames
        self._stage_latents(hn, arrays, n, count, frames)
        hn[count:count + n].view(np.int32)[:] = codes
        hn[count + n:].view(np.int32)[:] = 0
        torch = self.torch
        try:
            with torch.cuda.device(self.device):
                graph.replay()
                torch.cuda.current_stream(self.device).synchronize()
        except BaseException:
            self.out_buffers.release(lent)
            raise
        self._check_status(int(status_np[0]), lent)
        return self.out_buffers.lend(lent, lent[:n * HOP * frames].view(n, HOP * frames).numpy())

    def step(self, codes, arrays, frames):
        from ._native import check
        torch, lib = self.torch, self.lib
        n = len(arrays)
        count = n * 64 * frames
        shape = (n, HOP * frames)
        # The kernels write the audio straight into a lent pinned buffer when
        # it has a device address (no device-to-host copy after the step);
        # otherwise into device memory, downloaded afterwards.
        lent = self.out_buffers.acquire(n * HOP * frames)
        if lent is not None:
            fast = self.fast.get((n, frames, lent.data_ptr()))
            if fast is not None:
                return self._replay(fast, lent, codes, arrays, n, frames)
        with torch.cuda.device(self.device):
            # Latents (already in the staging buffer when the caller stacked
            # them there), slot codes and a zero status word: one upload.
            host = self._buffer("stage_host", (count + n + 1,), torch.float32, pinned=True)
            hn = host.numpy()
            self._stage_latents(hn, arrays, n, count, frames)
            hn[count:count + n].view(np.int32)[:] = codes
            hn[count + n:].view(np.int32)[:] = 0
            block = self._buffer("stage_dev", (count + n + 1,), torch.float32)
            z = block[:count]
            codes_dev = block[count:count + n]
            status = block[count + n:]
            target = self._mapped(lent) if lent is not None else None
            if target is None:
                if lent is not None:
                    self.out_buffers.release(lent)
                    lent = None
                audio = self._buffer("audio_dev", shape, torch.float32)
                target = audio.data_ptr()
            ws_bytes = int(lib.fav_plan_workspace_bytes(self.plan.handle, n, frames))
            ws = self._buffer("workspace", (ws_bytes,), torch.uint8)
            args = (self.plan.handle, self._ptr(self.pool), self.max_streams, self._ptr(codes_dev), n, frames,
                    self._ptr(z), ct.c_void_p(target), self._ptr(ws), ws_bytes, self._ptr(status))
            # Every buffer the graph reads or writes is part of its key (the
            # pinned staging buffer too: the graph's upload reads it).
            key = (n, frames, host.data_ptr(), z.data_ptr(), target, codes_dev.data_ptr(), ws.data_ptr())
            try:
                entry = self.graphs.get(key) if self.graphs_enabled else None
                if entry is None and self.graphs_enabled and key in self.graph_seen:
                    # The second step of a shape captures the upload, the
                    # kernels and the status download as one graph.
                    side = torch.cuda.Stream(self.device)
                    side.wait_stream(torch.cuda.current_stream(self.device))
                    graph = torch.cuda.CUDAGraph()
                    status_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
                    with torch.cuda.graph(graph, stream=side):
                        block.copy_(host, non_blocking=True)
                        check(lib, lib.fav_step(*args, ct.c_void_p(side.cuda_stream)))
                        status_host.copy_(status.view(torch.int32), non_blocking=True)
                    torch.cuda.current_stream(self.device).wait_stream(side)
                    entry = self.graphs[key] = (graph, status_host)
                    if lent is not None:
                        self.fast[(n, frames, lent.data_ptr())] = (hn, graph, status_host.numpy())
                if entry is not None:
                    entry[0].replay()
                    torch.cuda.current_stream(self.device).synchronize()
                    step_status = int(entry[1].item())
                else:
                    self.graph_seen.add(key)
                    block.copy_(host, non_blocking=True)
                    check(lib, lib.fav_step(*args, self._stream()))
                    step_status = None
            except BaseException:
                if lent is not None:
                    self.out_buffers.release(lent)
                raise
            if lent is None:
                if step_status is not None:
                    self._check_status(step_status, None)
                return self._download(audio, status)
            if step_status is None:
                self._finish(lent, status)
            else:
                self._check_status(step_status, lent)
            return self.out_buffers.lend(lent, lent[:n * HOP * frames].view(*shape).numpy())

    def decode_many(self, arrays, frames):
        from ._native import check
        torch, lib = self.torch, self.lib
        n = len(arrays)
        with torch.cuda.device(self.device):
            self.status.zero_()
            z = self._upload(arrays, frames)
            audio = self._buffer("batch_audio", (n, HOP * frames), torch.float32)
            chunk = min(self.chunk, frames)
            ws_bytes = int(lib.fav_plan_batch_workspace_bytes(self.plan.handle, n, chunk))
            ws = self._buffer("batch_ws", (ws_bytes,), torch.uint8)
            check(lib, lib.fav_decode_batch(self.plan.handle, self._ptr(z), n, frames, chunk, self._ptr(audio),
                                            self._ptr(ws), ws_bytes, self._ptr(self.status), self._stream()))
            return self._download(audio)

    def close(self):
        self.graphs = {}
        self.fast = {}
        if getattr(self, "plan", None) is not None:
            self.plan.close()


class CUDADecoder:
    """Immutable CUDA weights shared by independent, serialised streams."""

    def __init__(self, weights, info, mode, *, max_streams=256, device=0, batch_chunk_frames=128, backend=None,
                 precision=0):
        if mode not in ("batch", "streaming"):
            raise ValueError("mode must be batch or streaming")
        if type(max_streams) is not int or max_streams < 1:
            raise ValueError("max_streams must be a positive int")
        self.mode = mode
        self._max_streams = max_streams if mode == "streaming" else 1
        self._backend = backend if backend is not None else DeviceBackend(
            weights, max_streams=self._max_streams, device=device, batch_chunk_frames=batch_chunk_frames,
            precision=precision)
        self._lock = threading.Lock()
        self._free_slots = list(range(self._max_streams - 1, -1, -1))
        # Per-slot stream state (CUDAStream reads and writes it through its
        # slot), so a step over hundreds of streams builds its slot codes and
        # commits its histories with array operations.
        self._slot_parity = np.zeros(self._max_streams, np.int32)  # head table the history is read from
        self._slot_fresh = np.ones(self._max_streams, np.int32)    # 1: start from zero history
        self._slot_frames = np.zeros(self._max_streams, np.int64)  # frames decoded since (re)start
        self.state_bytes = STATE_BYTES
        self.info = {**info, "mode": mode, "state_bytes_per_stream": STATE_BYTES,
                     "state_device": "cuda", "output_device": "cpu", "output_ready": True,
                     "max_streams": self._max_streams,
                     "plan_device_bytes": getattr(self._backend, "plan_bytes", None)}

    # ------------------------------------------------------------ internals
    def _step(self, slots, arrays, frames):
        """One device step for the streams in ``slots`` (distinct); commits
        their histories only on success. Returns audio ``[n, 1, 1, 1920*frames]``."""
        n = len(slots)  # CUDAStream._code, over all streams at once
        codes = (slots << 2) | (self._slot_fresh[slots] * _FRESH) | self._slot_parity[slots]
        audio = self._backend.step(codes, arrays, frames)
        if (not isinstance(audio, np.ndarray) or audio.dtype != np.float32
                or audio.shape != (n, HOP * frames)):
            raise RuntimeError("CUDA model returned invalid audio")
        self._slot_parity[slots] ^= 1  # CUDAStream._commit, over all streams at once
        self._slot_fresh[slots] = 0
        self._slot_frames[slots] += frames
        return audio.reshape(n, 1, 1, HOP * frames)

    def _acquire_slot(self):
        with self._lock:
            if not self._free_slots:
                raise RuntimeError("All %d CUDA stream slots are in use; close a stream or raise max_streams"
                                   % self._max_streams)
            slot = self._free_slots.pop()
            self._slot_parity[slot] = 0
            self._slot_fresh[slot] = 1
            self._slot_frames[slot] = 0
            return slot

    def _release_slot(self, slot):
        with self._lock:
            self._free_slots.append(slot)

    # ------------------------------------------------------------ public API
    def prepare(self):
        """Warm the 1- and 2-frame step shapes without advancing any live stream."""
        if self.mode == "streaming":
            for frames in (1, 2):
                with self.stream() as s:
                    s.decode_chunk(np.zeros((1, 64, frames), np.float32))
        return self

    def decode(self, latents):
        """Decode an independent sequence in batch mode, starting with zero history."""
        if self.mode != "batch":
            raise RuntimeError("Use decoder.stream() for stateful streaming")
        latents = _latents(latents)
        if not latents.shape[2]:
            return np.empty((1, 1, 0), dtype=np.float32)
        return self.decode_many([latents])[0]

    def decode_many(self, clips):
        """Batch-decode equal-length clips ``[1,64,L]`` together (one launch per layer per chunk)."""
        if self.mode != "batch":
            raise RuntimeError("Use decoder.stream() for stateful streaming")
        clips = [_latents(c) for c in clips]
        if not clips:
            return []
        frames = clips[0].shape[2]
        if any(c.shape[2] != frames for c in clips):
            raise ValueError("decode_many requires clips of equal length")
        if not frames:
            return [np.empty((1, 1, 0), dtype=np.float32) for _ in clips]
        with self._lock:
            audio = self._backend.decode_many(clips, frames)
        if (not isinstance(audio, np.ndarray) or audio.dtype != np.float32
                or audio.shape != (len(clips), HOP * frames)):
            raise RuntimeError("CUDA model returned invalid audio")
        return [audio[i].reshape(1, 1, HOP * frames) for i in range(len(clips))]

    def stream(self):
        if self.mode != "streaming":
            raise RuntimeError("Load mode='streaming' to create an audio stream")
        return CUDAStream(self)

    def decode_streams(self, streams, chunks):
        """Decode one chunk for each of ``streams`` in a single step.

        All chunks must have the same frame count; each stream's history
        advances only if the whole step succeeds. Returns the audio as one
        float32 array ``[n, 1, 1, 1920*L]``; row i (``[1, 1, 1920*L]``) belongs
        to ``streams[i]``.
        """
        if self.mode != "streaming":
            raise RuntimeError("Load mode='streaming' to create an audio stream")
        if len(streams) != len(chunks):
            raise ValueError("One chunk per stream required")
        n = len(streams)
        if not n:
            _latents_step(chunks)
            return np.empty((0, 1, 1, 0), dtype=np.float32)
        if any(d is not self for d in set(map(_DECODER, streams))):
            raise ValueError("Stream belongs to another decoder")
        slots = np.fromiter(map(_SLOT, streams), np.int32, n)
        seen = np.zeros(self._max_streams, np.bool_)
        seen[slots] = True
        if int(seen.sum()) != n and len(set(map(id, streams))) != n:
            raise ValueError("A stream may appear only once per step")
        # Stream locks in one global (slot) order, so concurrent steps over
        # overlapping streams cannot deadlock.
        locks = list(map(_LOCK, map(streams.__getitem__, np.argsort(slots, kind="stable").tolist())))
        _drain(map(_LOCK_ACQUIRE, locks))
        try:
            if any(map(_CLOSED, streams)):  # (a closed stream's slot may belong to a live one)
                next(s for s in streams if s._closed)._check_open()
            with self._lock:
                # Validated (and stacked straight into the backend's upload
                # buffer) before any device work.
                stacked = _latents_step(chunks, getattr(self._backend, "stage", None))
                frames = stacked.shape[2]
                if not frames:
                    return np.empty((n, 1, 1, 0), dtype=np.float32)
                return self._step(slots, stacked, frames)
        finally:
            _drain(map(_LOCK_RELEASE, reversed(locks)))

    def close(self):
        close = getattr(self._backend, "close", None)
        if close:
            close()


class CUDAStream:
    """Per-utterance device history; all returned NumPy audio is ready to use."""

    def __init__(self, decoder):
        self._decoder = decoder
        self._lock = threading.Lock()
        self._slot = decoder._acquire_slot()
        self._closed = False
        self._frames_at_close = 0

    # The stream's state lives in its decoder's per-slot arrays.
    @property
    def frames_decoded(self):
        return self._frames_at_close if self._closed else int(self._decoder._slot_frames[self._slot])

    @property
    def _parity(self):
        return int(self._decoder._slot_parity[self._slot])

    @property
    def _fresh(self):
        return bool(self._decoder._slot_fresh[self._slot])

    def _code(self):
        return (self._slot << 2) | (_FRESH if self._fresh else 0) | self._parity

    def _check_open(self):
        if self._closed:
            raise RuntimeError("Decoder stream is closed; create a new stream")

    def decode_chunk(self, latents):
        """Decode fp32 ``[1,64,L]`` new frames; failures leave the history intact."""
        latents = _latents(latents)
        with self._lock:
            self._check_open()
            if not latents.shape[2]:
                return np.empty((1, 1, 0), dtype=np.float32)
            with self._decoder._lock:
                return self._decoder._step(np.array([self._slot], np.int32), latents, latents.shape[2])[0]

    def reset(self):
        with self._lock:
            self._check_open()
            self._decoder._slot_fresh[self._slot] = 1
            self._decoder._slot_frames[self._slot] = 0

    def flush(self):
        with self._lock:
            self._check_open()
            return np.empty((1, 1, 0), dtype=np.float32)

    def close(self):
        with self._lock:
            if not self._closed:
                self._frames_at_close = self.frames_decoded
                self._closed = True
                self._decoder._release_slot(self._slot)

    def __enter__(self):
        with self._lock:
            self._check_open()
        return self

    def __exit__(self, *exc):
        self.close()
