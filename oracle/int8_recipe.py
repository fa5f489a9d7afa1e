"""Restatement of the reference W8A8 matrix recipe (test infrastructure).

Follows ``experiments/intel-precision/native/precision.cpp`` (scalar backend 0):

* ``scale_of`` (``precision.cpp:88-92``): ``mx == 0 -> 1``; ``s = mx/127``; a
  non-positive (underflowed) ``s`` falls back to ``mx``.
* ``quantize`` (``:82-87``): ``clamp(v/scale, -127, 127)`` in fp32, then
  round-half-to-even.
* weights: one scale per matrix row (``ip_create``, ``:370-376``);
  activations: one scale per time column, reduced across K (``ip_prepare``,
  ``:395-415``).
* product: exact integer dot, ``float(dot) * (s_w[m] * s_x[t])`` (``scalar``,
  ``:242-247``).

``Int8RecipeDecoder`` applies the recipe where the reference's ``int8_large``
variant does (``experiments/intel-precision/tools/rewrite.py:19-42``): every
matrix with ``min(rows, cols) >= 128``. For this decoder that is the split
transposed-conv projections of stages 0-4 (rows ``(o, phase)``, one matrix per
tap, ``graph/upsampling.py:122-127``) and the residual 1x1 projections of
stages 0-3. Snake, depthwise, bias/residual, the stem 1x1 (K=64), stage 4-5
residuals, stage 5 transposed conv and the final conv stay fp32.
"""
from __future__ import annotations

import numpy as np
import torch

from . import exact
from .decoder import Decoder, RATES

INT8_MIN_DIM = 128


def scale_of(mx):
    """Vectorised ``precision.cpp:88-92``."""
    mx = np.asarray(mx, np.float32)
    s = (mx / np.float32(127)).astype(np.float32)
    return np.where(mx == 0, np.float32(1), np.where(s > 0, s, mx)).astype(np.float32)


def quantize(v, scale):
    """Vectorised ``precision.cpp:82-87``: clamp then round half to even."""
    q = np.clip((np.asarray(v, np.float32) / scale).astype(np.float32), -127, 127)
    return np.rint(q).astype(np.int32)


def quantize_rows(w):
    """Per-row weight quantisation (``ip_create``): returns (q [M,K] int32, s [M] fp32)."""
    w = np.asarray(w, np.float32)
    s = scale_of(np.max(np.abs(w), axis=1)) if w.shape[1] else np.ones(w.shape[0], np.float32)
    return quantize(w, s[:, None]), s


def quantize_columns(x):
    """Per-time-column activation quantisation (``ip_prepare``): (q [K,T], s [T])."""
    x = np.asarray(x, np.float32)
    s = scale_of(np.max(np.abs(x), axis=0)) if x.shape[0] else np.ones(x.shape[1], np.float32)
    return quantize(x, s[None, :]), s


def w8a8_matmul(w, x):
    """``y[M,T] = float(int dot) * (s_w * s_x)``, bit-exact to ``ip_run_rows`` backend 0."""
    qw, sw = quantize_rows(w)
    qx, sx = quantize_columns(x)
    dot = qw.astype(np.int64) @ qx.astype(np.int64)
    assert np.all(np.abs(dot) < 2**31)
    scale = (sw[:, None] * sx[None, :]).astype(np.float32)
    return (dot.astype(np.float32) * scale).astype(np.float32)


def selected_matrices():
    """Names of the projections the ``int8_large`` recipe quantises."""
    names = []
    cin = 2048
    for i, s in enumerate(RATES):
        cout = cin // 2
        if min(cout * s, cin) >= INT8_MIN_DIM:
            names.append(f"stage{i}.transpose")
        if cout >= INT8_MIN_DIM:
            names += [f"stage{i}.residual{j}.pointwise" for j in range(3)]
        cin = cout
    return names


class Int8RecipeDecoder(Decoder):
    """fp32 oracle decoder with the W8A8 recipe on the ``int8_large`` matrices.

    The transposed conv uses the split-projection lowering the CPU recipe
    quantises (``graph/upsampling.py:100-127``): ``current = W_cur @ x`` and
    ``previous = W_prev @ [history, x]`` shifted one frame, then
    ``(current + previous) + bias``.
    """

    def __init__(self, weights):
        super().__init__(weights)
        self.selected = set(selected_matrices())

    # The fp32 layers around the quantised projections run in one fixed
    # operation order (``oracle.exact``), the order the CUDA int8 path uses.
    def snake(self, x, alpha, reciprocal):
        return exact.snake_exact(x, alpha, reciprocal)

    def depthwise(self, x, history, weight, bias, dilation):
        return exact.depthwise_exact(x, history, weight, bias, dilation)

    def stem_pointwise(self, x):
        return exact.pointwise_exact(x, self.w["pointwise.weight"], self.w["pointwise.bias"])

    def transpose(self, i, x, history):
        if f"stage{i}.transpose" not in self.selected:
            return super().transpose(i, x, history)
        s = RATES[i]
        weight = self.w[f"stage{i}.transpose.weight"].numpy()
        bias = self.w[f"stage{i}.transpose.bias"].numpy()
        cin, cout, _ = weight.shape
        length = x.shape[-1]
        if length == 0:
            return x.new_empty((1, cout, 0)), history.clone()
        cur_w = weight[:, :, :s].transpose(1, 2, 0).reshape(cout * s, cin)
        prev_w = weight[:, :, s:].transpose(1, 2, 0).reshape(cout * s, cin)
        joined = torch.cat((history, x), dim=-1)[0].numpy()
        current = w8a8_matmul(cur_w, joined[:, 1:])
        previous = w8a8_matmul(prev_w, joined[:, :-1])
        phase = (current + previous).reshape(cout, s, length)
        y = phase.transpose(0, 2, 1).reshape(1, cout, length * s) + bias[None, :, None]
        return torch.from_numpy(np.ascontiguousarray(y, np.float32)), x[..., -1:].clone()

    def residual_pointwise(self, i, j, h):
        name = f"stage{i}.residual{j}.pointwise"
        if name not in self.selected:
            return super().residual_pointwise(i, j, h)
        weight = self.w[name + ".weight"].numpy()[:, :, 0]
        bias = self.w[name + ".bias"].numpy()
        y = w8a8_matmul(weight, h[0].numpy()) + bias[:, None]
        return torch.from_numpy(np.ascontiguousarray(y[None], np.float32))
