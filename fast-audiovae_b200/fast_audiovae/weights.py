"""AudioVAE2 decoder coefficients: architecture constants and a seeded initialiser.

The decoder graph follows the original export that the reference pins
(``src/fast_audiovae/mps_decoder.py:190-286`` in bevenky/fast-audiovae):

* stem: depthwise causal conv, 64 channels, k=7, d=1 (``mps_decoder.py:251``),
  then a 1x1 conv 64->2048 (``:252``);
* six up-stages with rates (8, 6, 5, 2, 2, 2) and channels 2048 -> 32
  (``:167``, ``:253-273``). Each stage is a per-channel affine ``x*scale+offset``
  (``:144-147``), Snake, a causal ConvTranspose1d with k=2s (``:263``) and three
  residual units at dilations 1, 3, 9, each Snake -> depthwise k=7 -> Snake ->
  1x1 -> + skip (``:264-271``);
* final: Snake(32) -> causal conv 32->1, k=7 -> tanh (``:274-275``, ``:321-322``).

The pinned ONNX export (trained weights) is not available, so coefficients come
from a variance-controlled seeded initialiser: Kaiming-normal style
``std = 1/sqrt(fan_in)`` with weight-norm folded, biases ``U(-0.01, 0.01)``,
Snake ``alpha ~ U(0.5, 1.5)`` with the stored reciprocal ``1/(alpha + 1e-9)``,
affine ``scale ~ U(0.9, 1.1)`` and ``offset ~ U(-0.01, 0.01)``. Three scale
corrections keep the random network out of tanh saturation: the transposed
convolutions use ``fan_in = 2*C_in`` (each output sees two taps), the eighteen
residual 1x1 weights are scaled by 0.1 and the final conv by 0.25.
"""
from __future__ import annotations

import numpy as np

SAMPLE_RATE = 48000
HOP_SAMPLES = 1920
LATENT_CHANNELS = 64
STEM_CHANNELS = 2048
RATES = (8, 6, 5, 2, 2, 2)
DILATIONS = (1, 3, 9)
FINAL_CHANNELS = 32
KERNEL = 7


def stage_channels(index):
    """(C_in, C_out) of up-stage ``index``."""
    return STEM_CHANNELS >> index, STEM_CHANNELS >> (index + 1)


def state_shapes():
    """The 26 causal histories in reference order (``mps_decoder.py:174-181``).

    Each history holds the most recent *inputs* of one causal operator, so the
    shapes are ``(1, channels, rows)`` exactly as the reference declares them.
    """
    shapes = {"stem.history": (1, LATENT_CHANNELS, 6)}
    for i in range(len(RATES)):
        cin, cout = stage_channels(i)
        shapes[f"stage{i}.transpose.history"] = (1, cin, 1)
        for j, d in enumerate(DILATIONS):
            shapes[f"stage{i}.residual{j}.history"] = (1, cout, 6 * d)
    shapes["final.history"] = (1, FINAL_CHANNELS, 6)
    return shapes


STATE_BYTES_FP32 = sum(int(np.prod(s)) * 4 for s in state_shapes().values())
assert len(state_shapes()) == 26 and STATE_BYTES_FP32 == 647424


def weight_shapes():
    """Canonical coefficient names and shapes, in generation order."""
    shapes = {
        "stem.weight": (LATENT_CHANNELS, 1, KERNEL),
        "stem.bias": (LATENT_CHANNELS,),
        "pointwise.weight": (STEM_CHANNELS, LATENT_CHANNELS, 1),
        "pointwise.bias": (STEM_CHANNELS,),
    }
    for i, s in enumerate(RATES):
        cin, cout = stage_channels(i)
        p = f"stage{i}."
        shapes[p + "scale"] = (cin,)
        shapes[p + "offset"] = (cin,)
        shapes[p + "snake.alpha"] = (cin,)
        shapes[p + "snake.reciprocal"] = (cin,)
        shapes[p + "transpose.weight"] = (cin, cout, 2 * s)
        shapes[p + "transpose.bias"] = (cout,)
        for j in range(len(DILATIONS)):
            r = f"{p}residual{j}."
            shapes[r + "pre.alpha"] = (cout,)
            shapes[r + "pre.reciprocal"] = (cout,)
            shapes[r + "depthwise.weight"] = (cout, 1, KERNEL)
            shapes[r + "depthwise.bias"] = (cout,)
            shapes[r + "post.alpha"] = (cout,)
            shapes[r + "post.reciprocal"] = (cout,)
            shapes[r + "pointwise.weight"] = (cout, cout, 1)
            shapes[r + "pointwise.bias"] = (cout,)
    shapes["final.snake.alpha"] = (FINAL_CHANNELS,)
    shapes["final.snake.reciprocal"] = (FINAL_CHANNELS,)
    shapes["final.weight"] = (1, FINAL_CHANNELS, KERNEL)
    shapes["final.bias"] = (1,)
    return shapes


def _fan_in_and_gain(name, shape):
    if name == "stem.weight" or name.endswith("depthwise.weight"):
        return KERNEL, 1.0
    if name.endswith("transpose.weight"):
        return 2 * shape[0], 1.0
    if name.endswith("pointwise.weight"):
        return shape[1], (0.1 if ".residual" in name else 1.0)
    if name == "final.weight":
        return shape[1] * KERNEL, 0.25
    raise KeyError(name)


def seeded_weights(seed=0):
    """Deterministic fp32 coefficients for ``seed`` (dict name -> ndarray)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in weight_shapes().items():
        if name.endswith(".reciprocal"):
            alpha = out[name[: -len("reciprocal")] + "alpha"]
            out[name] = (np.float32(1.0) / (alpha + np.float32(1e-9))).astype(np.float32)
        elif name.endswith(".alpha"):
            out[name] = rng.uniform(0.5, 1.5, shape).astype(np.float32)
        elif name.endswith(".bias"):
            out[name] = rng.uniform(-0.01, 0.01, shape).astype(np.float32)
        elif name.endswith(".scale"):
            out[name] = rng.uniform(0.9, 1.1, shape).astype(np.float32)
        elif name.endswith(".offset"):
            out[name] = rng.uniform(-0.01, 0.01, shape).astype(np.float32)
        else:
            fan_in, gain = _fan_in_and_gain(name, shape)
            std = gain / np.sqrt(fan_in)
            out[name] = (rng.standard_normal(shape) * std).astype(np.float32)
    return out


def seeded_latents(seed, frames):
    """Latents ``[1, 64, frames]`` ~ N(0, 1) in fp32 from ``default_rng(seed)``."""
    return np.random.default_rng(seed).standard_normal((1, LATENT_CHANNELS, frames), np.float32)


def validate_weights(weights):
    """Raise ``ValueError`` unless ``weights`` holds every finite fp32 coefficient."""
    shapes = weight_shapes()
    if not isinstance(weights, dict) or set(weights) != set(shapes):
        raise ValueError("Weights must hold exactly the decoder's coefficients")
    for name, shape in shapes.items():
        value = weights[name]
        if (not isinstance(value, np.ndarray) or value.dtype != np.float32
                or value.shape != shape or not np.isfinite(value).all()):
            raise ValueError("Finite fp32 coefficient of shape %s required: %s" % (shape, name))
