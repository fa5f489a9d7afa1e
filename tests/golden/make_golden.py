"""Generate the golden vectors that pin the oracle to the reference.

Run in a checkout where the reference tree is present (it is read from
``oracle.reference.REFERENCE_ROOT``) after
``make -C oracle ref``:

    python tests/golden/make_golden.py

Outputs (small ``.npz`` files next to this script):

* ``decoder_seed0.npz``: the reference's own fp32 decoder
  (``src/fast_audiovae/mps_decoder.py`` ``MPSModel``, CPU) on the seeded
  coefficients (``seeded_weights(0)``): batch audio for latents seed 0 with 3 and
  25 frames, a streamed decode of the 25 frames in chunks (1, 7, 2, 3, 11) and
  five of the 26 histories after the 3-frame decode.
* ``int8_core.npz``: the reference int8 core (``precision.cpp``, backend 0,
  compiled from its source by ``oracle/Makefile``) on the small shapes of its
  own check (``experiments/intel-precision/native/check_micro.py:80-87``), the
  full-range signedness cases and the exact-zero case (``:108-114``).
* ``int8_decoder_seed0.npz``: the int8-recipe decoder with every W8A8 product
  computed by the compiled reference core, latents seed 0, 3 frames (the fp32
  layers around the products in ``oracle.exact``'s operation order).
* ``elementwise.npz``: the reference x86 C kernels (``native_kernels.c``,
  scalar libm sine) for fused Snake -> DW7 -> Snake at dilations 1/3/9 and
  ``skip + (product + bias)``.
"""
from __future__ import annotations

import ctypes as ct
import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "fast-audiovae_b200"))
sys.path.insert(0, str(ROOT))

from fast_audiovae import weights as W  # noqa: E402
from oracle import int8_recipe, reference  # noqa: E402


def weights_digest(weights):
    h = hashlib.sha256()
    for name in W.weight_shapes():
        h.update(name.encode())
        h.update(np.ascontiguousarray(weights[name], np.float32).tobytes())
    return h.hexdigest()


def decoder_golden():
    torch.set_num_threads(1)
    w = W.seeded_weights(0)
    model = reference.reference_decoder(w)
    out = {"weights_sha256": np.array(weights_digest(w))}
    z3 = W.seeded_latents(0, 3)
    with torch.inference_mode():
        audio3, states = model.decode(torch.from_numpy(z3.copy()), {})
        out["z3"], out["audio3"] = z3, audio3.numpy()
        for name in ("stem.history", "stage0.transpose.history", "stage3.residual1.history",
                     "stage5.residual2.history", "final.history"):
            out["state3/" + name] = states[name].numpy()
        z25 = W.seeded_latents(0, 25)
        audio25, _ = model.decode(torch.from_numpy(z25.copy()), {})
        out["z25"], out["audio25"] = z25, audio25.numpy()
        parts, hist, start, k = [], {}, 0, 0
        pattern = (1, 7, 2, 3, 11)
        while start < 25:
            end = min(25, start + pattern[k % len(pattern)])
            piece, hist = model.decode(torch.from_numpy(z25[..., start:end].copy()), hist)
            parts.append(piece.numpy())
            start, k = end, k + 1
        out["stream25_uneven"] = np.concatenate(parts, axis=-1)
    np.savez_compressed(HERE / "decoder_seed0.npz", **out)


def int8_core_golden():
    rng = np.random.default_rng(20260908)
    out = {}
    shapes = [(1, 1, 0), (1, 1, 1), (3, 5, 7), (17, 31, 16), (32, 32, 33), (64, 64, 65), (3, 2048, 17),
              (257, 64, 1)]
    for i, (m, k, t) in enumerate(shapes):
        w = (rng.normal(size=(m, k)) * .2).astype(np.float32)
        x = (rng.normal(size=(k, t)) * .2).astype(np.float32)
        w *= np.linspace(.2, 3, m, dtype=np.float32)[:, None]
        if t:
            x *= np.linspace(.1, 5, t, dtype=np.float32)[None, :]
        out[f"case{i}/w"], out[f"case{i}/x"] = w, x
        out[f"case{i}/y"] = reference.precision_matmul(w, x)
    i = len(shapes)
    for sign_w, sign_x in ((1, 1), (1, -1), (-1, 1), (-1, -1)):
        w = np.full((16, 128), sign_w * 127, dtype=np.float32)
        x = np.full((128, 17), sign_x * 127, dtype=np.float32)
        out[f"case{i}/w"], out[f"case{i}/x"], out[f"case{i}/y"] = w, x, reference.precision_matmul(w, x)
        i += 1
    w = np.zeros((3, 7), np.float32)
    x = np.zeros((7, 5), np.float32)
    w[1] = [-3, -2, -1, 0, 1, 2, 3]
    x[:, 2] = [-3, -2, -1, 0, 1, 2, 3]
    out[f"case{i}/w"], out[f"case{i}/x"], out[f"case{i}/y"] = w, x, reference.precision_matmul(w, x)
    np.savez_compressed(HERE / "int8_core.npz", **out)


def int8_decoder_golden():
    torch.set_num_threads(1)
    w = W.seeded_weights(0)
    z = W.seeded_latents(0, 3)
    saved = int8_recipe.w8a8_matmul
    int8_recipe.w8a8_matmul = reference.precision_matmul
    try:
        audio = int8_recipe.Int8RecipeDecoder(w).decode_numpy(z)
    finally:
        int8_recipe.w8a8_matmul = saved
    np.savez_compressed(HERE / "int8_decoder_seed0.npz", weights_sha256=np.array(weights_digest(w)), z=z,
                        audio=audio)


def elementwise_golden():
    lib = reference.native_library()
    P = ct.POINTER(ct.c_float)
    ptr = lambda a: a.ctypes.data_as(P)
    rng = np.random.default_rng(11)
    out = {}
    B, C, T = 1, 8, 40
    for d in (1, 3, 9):
        x = rng.normal(0, 1.5, (B, C, T)).astype(np.float32)
        w = (rng.normal(0, 0.4, (C, 7))).astype(np.float32)
        b = rng.uniform(-0.01, 0.01, C).astype(np.float32)
        a1 = rng.uniform(0.5, 1.5, C).astype(np.float32)
        r1 = (1 / (a1 + np.float32(1e-9))).astype(np.float32)
        a2 = rng.uniform(0.5, 1.5, C).astype(np.float32)
        r2 = (1 / (a2 + np.float32(1e-9))).astype(np.float32)
        y = np.zeros_like(x)
        st = lib.ncc_snake_dw7_snake_f32(ptr(x), ptr(w), ptr(b), ptr(a1), ptr(r1), ptr(a2), ptr(r2), ptr(y),
                                         B, C, T, d, 1, 1)
        assert st == 0, st
        for key, value in dict(x=x, w=w, b=b, a1=a1, r1=r1, a2=a2, r2=r2, y=y).items():
            out[f"sds{d}/{key}"] = value
    prod = rng.normal(0, 1, (1, 8, 33)).astype(np.float32)
    skip = rng.normal(0, 1, (1, 8, 33)).astype(np.float32)
    bias = rng.normal(0, 1, 8).astype(np.float32)
    y = np.zeros_like(prod)
    assert lib.ncc_bias_residual_f32(ptr(prod), ptr(bias), ptr(skip), ptr(y), 1, 8, 33, 1, 1) == 0
    out.update({"br/product": prod, "br/skip": skip, "br/bias": bias, "br/y": y})
    np.savez_compressed(HERE / "elementwise.npz", **out)


if __name__ == "__main__":
    if not reference.reference_available():
        sys.exit("reference sources not found")
    decoder_golden()
    int8_core_golden()
    int8_decoder_golden()
    elementwise_golden()
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)
