"""AudioVAE2 decoder on NVIDIA B200 (sm_100a): the reference's facade for device="cuda".

Mirrors ``src/fast_audiovae/__init__.py:11-14`` and ``automatic.py:274-284`` of
bevenky/fast-audiovae: ``load(mode=..., threads=..., device=..., **options)``
returns a decoder with ``.decode`` (batch), ``.stream()`` (streaming) and
``.info``. Only ``device="cuda"`` is provided here; the reference's CPU/ONNX
and Apple routes are outside this package.

Coefficients: the reference loads a checksum-pinned ONNX export
(``assets.py:6-11``); ``load(source="<dir>/audio_vae_decoder.onnx")`` reads it
the same way (``fast_audiovae.onnx_import``, no ``onnx`` package needed; the
pinned digests are required unless ``pinned_export=False``). ``load`` also
takes ``weights=`` (a coefficient dict, names from
``fast_audiovae.weights.weight_shapes()``), ``source=`` an ``.npz`` file with
those names, or, by default, the seeded random init of
``fast_audiovae.weights.seeded_weights(weight_seed)``.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

from . import weights
from . import weights as _coeffs

__all__ = ["load", "setup", "weights"]

_MODES = {"batch": "batch", "streaming": "streaming", "stream": "streaming"}


def _options(mode, threads, device):
    if mode not in _MODES:
        raise ValueError("mode must be batch or streaming")
    if device != "cuda":
        raise ValueError("device must be cuda: this package provides the B200 CUDA decoder only")
    if type(threads) is not int or threads != 1:
        raise ValueError("CUDA decoding requires threads=1; CPU worker counts do not control the GPU")
    return _MODES[mode]


# Precisions (values of the C ABI's fav_precision).
PRECISIONS = {
    "bf16": (0, "split-bf16 transposed/stem projections, f16 residual projections, fp32 accumulate"),
    "int8": (1, "W8A8 int8 recipe on the projections with min(rows, cols) >= 128 (s8 tensor cores, per-row weight "
                "and per-time-step activation scales, s32 accumulate); other layers as bf16"),
}


def _coefficients(weights_arg, source, weight_seed, pinned=True):
    if weights_arg is not None and source is not None:
        raise ValueError("Pass weights or source, not both")
    if weights_arg is not None:
        coeffs = {k: np.array(v, dtype=np.float32, copy=True) for k, v in weights_arg.items()}
        origin = "caller_coefficients"
    elif source is not None and str(source).endswith(".onnx"):
        from . import onnx_import
        coeffs = onnx_import.load_coefficients(Path(source).expanduser(), pinned=pinned)
        origin = "onnx:" + str(Path(source).expanduser().resolve()) + (" (pinned)" if pinned else "")
    elif source is not None:
        with np.load(Path(source).expanduser(), allow_pickle=False) as archive:
            coeffs = {k: np.array(archive[k], dtype=np.float32, copy=True) for k in archive.files}
        origin = "npz:" + str(Path(source).expanduser().resolve())
    else:
        coeffs = _coeffs.seeded_weights(weight_seed)
        origin = f"seeded_random_init(seed={weight_seed})"
    _coeffs.validate_weights(coeffs)
    return coeffs, origin


def setup(*, mode="streaming", threads=1, device="cuda", cache_dir=None, source=None, offline=False,
          prefer_custom=True, weights=None, weight_seed=0, precision="bf16", **_ignored):
    """Validate options and describe the selected route, without building a decoder.

    Mirrors ``gpu.setup_gpu`` (``gpu.py:55-95``): no decoder is instantiated and
    no inference runs. ``cache_dir``, ``offline`` and ``prefer_custom`` are CPU
    recipe options of the reference and have no effect on the CUDA route.
    """
    selected = _options(mode, threads, device)
    if precision not in PRECISIONS:
        raise ValueError("precision must be bf16 or int8")
    return {"device": "cuda", "backend": "cuda", "selected": "b200_tcgen05", "recipe": "b200_sm100a_v1",
            "precision": precision, "precision_detail": PRECISIONS[precision][1],
            "mode": selected, "threads": 1, "cpu_only": False, "fallback": False,
            "reason": "Explicit CUDA request", "sample_rate": _coeffs.SAMPLE_RATE,
            "latent_rate": 25, "latent_channels": 64, "samples_per_latent": _coeffs.HOP_SAMPLES,
            "source": str(source) if source is not None else None, "weight_seed": weight_seed}


def load(*, mode="streaming", threads=1, device="cuda", cache_dir=None, source=None, offline=False,
         prefer_custom=True, weights=None, weight_seed=0, max_streams=256, device_index=0, precision="bf16",
         pinned_export=True):
    """Load the CUDA decoder; ``mode="stream"`` is accepted as an alias of ``"streaming"``.

    ``precision="int8"`` runs the reference's W8A8 int8 recipe on its selected
    projections (experiments/intel-precision), the rest as ``"bf16"``.
    ``source`` may name the AudioVAE2 ONNX export (``*.onnx`` beside its
    ``.onnx.data``), read as ``MPSModel.from_onnx`` does (mps_decoder.py:190-286).
    """
    info = setup(mode=mode, threads=threads, device=device, cache_dir=cache_dir, source=source,
                 offline=offline, prefer_custom=prefer_custom, weight_seed=weight_seed, precision=precision)
    coeffs, origin = _coefficients(weights, source, weight_seed, pinned_export)
    from .cuda import CUDADecoder
    decoder = CUDADecoder(coeffs, {**info, "coefficient_source": origin}, info["mode"],
                          max_streams=max_streams, device=device_index, precision=PRECISIONS[precision][0])
    import torch
    props = torch.cuda.get_device_properties(decoder._backend.device)
    decoder.info.update(device_name=props.name, sm_count=props.multi_processor_count)
    if decoder.mode == "streaming":
        decoder.prepare()
    return decoder
