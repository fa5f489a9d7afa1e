"""fp32 restatement of the reference AudioVAE2 decoder (test infrastructure).

Follows ``src/fast_audiovae/mps_decoder.py`` of bevenky/fast-audiovae operation
by operation, in torch fp32 on the CPU, so that each rounding point of the
reference is kept:

* Snake: ``scaled=alpha*x; s=sin(scaled); sq=s*s; corr=r*sq; y=x+corr`` with the
  stored reciprocal ``r`` (``mps_decoder.py:44-50``).
* 1x1 conv: ``W @ x + b`` (``:61-62``).
* causal depthwise/regular conv: history concatenated on the left, history out
  = last ``6*d`` inputs (``:77-83``).
* causal ConvTranspose1d, polyphase: stage 0 "paired" (one reduction over
  ``[x_t; x_{t-1}]``), later stages split into two projections summed as
  ``cur + prev`` (``:96-121``); bias added once; history = last activated input.
* residual: ``x + (W @ h + b)`` (``:130-134``); stage affine ``x*scale`` then
  ``+offset`` (``:144-147``); final ``tanh`` (``:321-322``).

States use the reference names and shapes (``mps_decoder.py:174-181``).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

RATES = (8, 6, 5, 2, 2, 2)
DILATIONS = (1, 3, 9)
HOP = 1920


def snake(x, alpha, reciprocal):
    """``mps_decoder.py:44-50``; alpha/reciprocal are [C] tensors."""
    a = alpha.reshape(1, -1, 1)
    r = reciprocal.reshape(1, -1, 1)
    scaled = a * x
    sine = torch.sin(scaled)
    squared = sine * sine
    correction = r * squared
    return x + correction


def pointwise(x, weight, bias):
    """``mps_decoder.py:61-62``: ``mm(W[:, :, 0], x[0]) + b``."""
    return torch.mm(weight[:, :, 0], x[0]).unsqueeze(0) + bias[None, :, None]


def causal_conv(x, history, weight, bias, dilation=1, groups=1):
    """``mps_decoder.py:77-83``: returns (y, new history = last 6*d inputs)."""
    halo = 6 * dilation
    joined = torch.cat((history, x), dim=-1)
    if x.shape[-1] == 0:
        return x.new_empty((x.shape[0], weight.shape[0], 0)), history.clone()
    y = F.conv1d(joined, weight, bias, dilation=dilation, groups=groups)
    return y, joined[..., -halo:].clone()


def pack_transpose(weight, stride, paired):
    """Load-time packing of ``mps_decoder.py:99-105``."""
    cin, cout, _ = weight.shape
    if paired:
        current = weight[..., :stride].permute(1, 2, 0)
        previous = weight[..., stride:].permute(1, 2, 0)
        return torch.cat((current, previous), dim=-1).reshape(cout * stride, 2 * cin).contiguous()
    return weight.permute(1, 2, 0).reshape(cout * 2 * stride, cin).contiguous()


def causal_transpose(x, history, packed, bias, stride, paired):
    """``mps_decoder.py:107-121``: polyphase transposed conv, right-cropped."""
    length = x.shape[-1]
    channels = bias.shape[0]
    if length == 0:
        return x.new_empty((1, channels, 0)), history.clone()
    if paired:
        previous = torch.cat((history, x[..., :-1]), dim=-1)
        features = torch.cat((x[0], previous[0]), dim=0)
        y = torch.mm(packed, features).reshape(channels, stride, length)
    else:
        joined = torch.cat((history, x), dim=-1)
        projection = torch.mm(packed, joined[0]).reshape(channels, 2 * stride, length + 1)
        y = projection[:, :stride, 1:] + projection[:, stride:, :-1]
    y = y.permute(0, 2, 1).reshape(1, channels, length * stride)
    return (y + bias[None, :, None]).contiguous(), x[..., -1:].clone()


def state_shapes():
    shapes = {"stem.history": (1, 64, 6)}
    cin = 2048
    for i in range(len(RATES)):
        cout = cin // 2
        shapes[f"stage{i}.transpose.history"] = (1, cin, 1)
        for j, d in enumerate(DILATIONS):
            shapes[f"stage{i}.residual{j}.history"] = (1, cout, 6 * d)
        cin = cout
    shapes["final.history"] = (1, 32, 6)
    return shapes


class Decoder:
    """fp32 CPU decoder over a coefficient dict (names from the package's weights).

    ``matmul`` hooks let the int8 oracle replace selected projections; by
    default every projection is the fp32 ``torch.mm`` of the reference.
    """

    def __init__(self, weights, dtype=torch.float32):
        self.dtype = dtype
        self.w = {k: torch.from_numpy(np.array(v, copy=True)).to(dtype) for k, v in weights.items()}
        self.packed = {}
        for i, s in enumerate(RATES):
            self.packed[i] = pack_transpose(self.w[f"stage{i}.transpose.weight"], s, paired=(i == 0))
        self.state_shapes = state_shapes()

    def zero_states(self):
        return {k: torch.zeros(s, dtype=self.dtype) for k, s in self.state_shapes.items()}

    # Projection hooks (overridden by the int8 recipe oracle).
    def stem_pointwise(self, x):
        return pointwise(x, self.w["pointwise.weight"], self.w["pointwise.bias"])

    def transpose(self, i, x, history):
        s = RATES[i]
        return causal_transpose(x, history, self.packed[i], self.w[f"stage{i}.transpose.bias"], s, i == 0)

    def residual_pointwise(self, i, j, h):
        p = f"stage{i}.residual{j}.pointwise."
        return pointwise(h, self.w[p + "weight"], self.w[p + "bias"])

    # Elementwise and depthwise hooks (the int8 recipe oracle fixes their fp32 operation order).
    def snake(self, x, alpha, reciprocal):
        return snake(x, alpha, reciprocal)

    def depthwise(self, x, history, weight, bias, dilation):
        return causal_conv(x, history, weight, bias, dilation, x.shape[1])

    @torch.inference_mode()
    def decode(self, z, states=None, trace=None):
        """One step: ``z`` [1,64,T] (numpy or tensor) -> (audio [1,1,1920T], states).

        ``trace`` (a list) receives the 25 projection-layer outputs in order:
        stem 1x1, then per stage the transposed conv and the three residual units.
        """
        def keep(v):
            if trace is not None:
                trace.append(v.clone())
            return v
        w = self.w
        if isinstance(z, np.ndarray):
            z = torch.from_numpy(np.array(z, copy=True))
        z = z.to(self.dtype)
        history = self.zero_states() if not states else states
        if z.shape[-1] == 0:
            return z.new_empty((1, 1, 0)), {k: v.clone() for k, v in history.items()}
        out = {}
        x, out["stem.history"] = self.depthwise(z, history["stem.history"], w["stem.weight"], w["stem.bias"], 1)
        x = keep(self.stem_pointwise(x))
        for i in range(len(RATES)):
            p = f"stage{i}."
            x = x * w[p + "scale"].reshape(1, -1, 1)
            x = x + w[p + "offset"].reshape(1, -1, 1)
            key = p + "transpose.history"
            x, out[key] = self.transpose(i, self.snake(x, w[p + "snake.alpha"], w[p + "snake.reciprocal"]),
                                         history[key])
            keep(x)
            for j, d in enumerate(DILATIONS):
                r = f"{p}residual{j}."
                key = r[:-1] + ".history"
                before = self.snake(x, w[r + "pre.alpha"], w[r + "pre.reciprocal"])
                branch, out[key] = self.depthwise(before, history[key], w[r + "depthwise.weight"],
                                                  w[r + "depthwise.bias"], d)
                branch = self.snake(branch, w[r + "post.alpha"], w[r + "post.reciprocal"])
                x = keep(x + self.residual_pointwise(i, j, branch))
        before = self.snake(x, w["final.snake.alpha"], w["final.snake.reciprocal"])
        x, out["final.history"] = causal_conv(before, history["final.history"], w["final.weight"],
                                              w["final.bias"], 1, 1)
        return torch.tanh(x), out

    def decode_numpy(self, z):
        """Batch decode of a numpy [1,64,L] array to numpy audio [1,1,1920L] (fp32)."""
        audio, _ = self.decode(z)
        return audio.to(torch.float32).numpy()

    def stream_numpy(self, z, pattern):
        """Chunked streaming decode with carried history (``streaming.py:78-112``)."""
        states, parts, start, k = None, [], 0, 0
        while start < z.shape[-1]:
            end = min(z.shape[-1], start + pattern[k % len(pattern)])
            audio, states = self.decode(z[..., start:end], states)
            parts.append(audio.to(torch.float32).numpy())
            start, k = end, k + 1
        return np.concatenate(parts, axis=-1) if parts else np.empty((1, 1, 0), np.float32)


def discrepancy(reference, actual):
    """Waveform comparison of ``tools/validate_streaming.py:61-82``: max_abs, rmse, SNR, exact."""
    ref = np.asarray(reference, np.float64)
    err = np.asarray(actual, np.float64) - ref
    mse = float(np.mean(err * err)) if err.size else 0.0
    signal = float(np.mean(ref * ref)) if ref.size else 0.0
    return {
        "max_abs": float(np.max(np.abs(err))) if err.size else 0.0,
        "rmse": float(np.sqrt(mse)),
        "snr_db": float(10 * np.log10(signal / mse)) if mse > 0 and signal > 0 else float("inf"),
        "exact": bool(np.array_equal(np.asarray(reference, np.float32).view(np.uint32),
                                     np.asarray(actual, np.float32).view(np.uint32))),
    }
