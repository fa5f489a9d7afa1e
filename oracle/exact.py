"""fp32 operations in one fixed order, for the int8 recipe oracle (test infrastructure).

The reference's int8 recipe (experiments/intel-precision) quantises each
selected projection's input per time step; a quantised cascade is so
sensitive that two fp32 implementations of the surrounding layers which differ
in the last bit of one value end up ~38 dB apart after the five stages (one
ulp at the stem output; measured with this oracle). Parity with the recipe is
therefore checked against this oracle, whose fp32 layers around the quantised
projections are written as an explicit sequence of IEEE operations (no fused
multiply-add) that the CUDA int8 path executes in the same order:

* ``sin_cw``: sine by Cody-Waite argument reduction (W. J. Cody and W. Waite,
  Software Manual for the Elementary Functions, 1980) with pi/2 split in three
  parts, and Taylor polynomials of degree 11 (sine) and 12 (cosine) on
  [-pi/4, pi/4] evaluated by Horner's rule; within a few ulp of the true sine
  for the arguments Snake sees.
* ``snake_exact``: ``x + r * (s * s)``, ``s = sin_cw(alpha * x)``, rounding
  as ``mps_decoder.py:44-50`` (three products and one sum, each rounded).
* ``depthwise_exact``: causal depthwise conv k=7, taps summed oldest first,
  bias added last (``mps_decoder.py:65-83``).
* ``pointwise_exact``: the stem 1x1 projection, input channels summed in
  order, bias added last (``mps_decoder.py:53-62``).
"""
from __future__ import annotations

import numpy as np
import torch

F32 = np.float32


def _split_half_pi():
    """pi/2 = P1 + P2 + P3 with P1 and P2 of at most 15 significant bits, so
    k * P1 and k * P2 are exact in fp32 for |k| < 2^9."""
    half_pi = np.pi / 2

    def head(v, bits):
        m, e = np.frexp(v)
        return np.ldexp(np.trunc(m * 2.0 ** bits), e - bits)

    p1 = head(half_pi, 15)
    p2 = head(half_pi - p1, 15)
    p3 = half_pi - p1 - p2
    return F32(p1), F32(p2), F32(p3)


TWO_OVER_PI = F32(2 / np.pi)
P1, P2, P3 = _split_half_pi()
# Taylor coefficients of sin (odd) and cos (even), rounded to fp32.
S = [F32(-1 / 6), F32(1 / 120), F32(-1 / 5040), F32(1 / 362880), F32(-1 / 39916800)]
C = [F32(-1 / 2), F32(1 / 24), F32(-1 / 720), F32(1 / 40320), F32(-1 / 3628800), F32(1 / 479001600)]


def constants():
    """The constants as fp32 bit patterns (for the CUDA restatement's test)."""
    vals = {"two_over_pi": TWO_OVER_PI, "p1": P1, "p2": P2, "p3": P3}
    vals.update({f"s{2 * i + 3}": c for i, c in enumerate(S)})
    vals.update({f"c{2 * i + 2}": c for i, c in enumerate(C)})
    return {k: int(np.asarray(v, F32).view(np.uint32)) for k, v in vals.items()}


def sin_cw(x):
    """Elementwise sine of a float32 tensor, fp32 operations in a fixed order."""
    x = x.to(torch.float32)
    k = torch.round(x * float(TWO_OVER_PI))          # half to even
    r = ((x - k * float(P1)) - k * float(P2)) - k * float(P3)
    r2 = r * r
    ps = r2 * float(S[4])
    for c in (S[3], S[2], S[1], S[0]):
        ps = r2 * (ps + float(c))
    sin_r = r + r * ps
    pc = r2 * float(C[5])
    for c in (C[4], C[3], C[2], C[1], C[0]):
        pc = r2 * (pc + float(c))
    cos_r = 1.0 + pc
    q = k.to(torch.int32) & 3
    out = torch.where(q == 0, sin_r, torch.where(q == 1, cos_r, torch.where(q == 2, -sin_r, -cos_r)))
    return out.to(torch.float32)


def snake_exact(x, alpha, reciprocal):
    a = alpha.reshape(1, -1, 1)
    r = reciprocal.reshape(1, -1, 1)
    s = sin_cw(a * x)
    return x + r * (s * s)


def depthwise_exact(x, history, weight, bias, dilation):
    """Causal depthwise conv k=7: returns (y, new history = last 6*d inputs)."""
    halo = 6 * dilation
    joined = torch.cat((history, x), dim=-1)
    length = x.shape[-1]
    if length == 0:
        return x.new_empty(x.shape), history.clone()
    w = weight[:, 0, :]  # [C, 7]
    y = w[:, 0:1] * joined[0, :, 0:length]
    for j in range(1, 7):
        y = y + w[:, j:j + 1] * joined[0, :, j * dilation:j * dilation + length]
    y = y + bias[:, None]
    return y.unsqueeze(0), joined[..., -halo:].clone()


def pointwise_exact(x, weight, bias):
    """1x1 projection, input channels summed in order, then the bias."""
    w = weight[:, :, 0]  # [N, K]
    xs = x[0]            # [K, T]
    y = w[:, 0:1] * xs[0:1, :]
    for k in range(1, w.shape[1]):
        y = y + w[:, k:k + 1] * xs[k:k + 1, :]
    return (y + bias[:, None]).unsqueeze(0)
