"""The int8 recipe restatement against the compiled reference core (CPU).

Golden vectors were produced by ``experiments/intel-precision/native/precision.cpp``
(backend 0) compiled from the reference source; the restatement must match
them bit for bit. Where the compiled reference is present, it is also
checked live on fresh random shapes.
"""
import numpy as np
import pytest

from fast_audiovae import weights as W
from oracle import int8_recipe as R
from oracle import reference


def test_w8a8_matches_reference_core_bitwise(golden):
    g = golden("int8_core.npz")
    cases = sorted({k.split("/")[0] for k in g})
    assert len(cases) == 13
    for case in cases:
        y = R.w8a8_matmul(g[case + "/w"], g[case + "/x"])
        assert y.shape == g[case + "/y"].shape
        assert np.array_equal(y.view(np.uint32), g[case + "/y"].view(np.uint32)), case


def test_scale_and_rounding_rules():
    """``precision.cpp:82-92``: zero -> 1, subnormal fallback, half to even."""
    assert R.scale_of(np.float32(0)) == 1
    tiny = np.float32(1e-44)
    assert R.scale_of(tiny) == tiny
    q = R.quantize(np.array([0.5, 1.5, 2.5, -0.5, -1.5, 200, -200], np.float32), np.float32(1))
    assert q.tolist() == [0, 2, 2, 0, -2, 127, -127]


def test_selected_matrices_follow_int8_large_rule():
    names = R.selected_matrices()
    assert names.count("stage0.transpose") == 1
    assert "stage5.transpose" not in names and "stage4.transpose" in names
    assert "stage3.residual2.pointwise" in names and "stage4.residual0.pointwise" not in names
    assert sum(n.endswith("pointwise") for n in names) == 12 and sum(n.endswith("transpose") for n in names) == 5


def test_int8_decoder_matches_reference_core_decoder(golden):
    g = golden("int8_decoder_seed0.npz")
    audio = R.Int8RecipeDecoder(W.seeded_weights(0)).decode_numpy(g["z"])
    assert np.array_equal(audio.view(np.uint32), g["audio"].view(np.uint32))


@pytest.mark.skipif(not (reference.REF_LIB_DIR / "libprecision_ref.so").is_file(),
                    reason="compiled reference int8 core not built here")
def test_w8a8_matches_live_reference_core():
    rng = np.random.default_rng(5)
    for m, k, t in [(7, 9, 11), (128, 256, 33), (1, 1, 5), (40, 2048, 3)]:
        w = rng.normal(0, 0.3, (m, k)).astype(np.float32)
        x = rng.normal(0, 2.0, (k, t)).astype(np.float32)
        x[:, 0] = 0
        a, b = R.w8a8_matmul(w, x), reference.precision_matmul(w, x)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
