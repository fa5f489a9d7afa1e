"""The oracle against the reference: golden vectors and known-answer tests (CPU).

Golden vectors come from the reference's own decoder (``tests/golden/make_golden.py``).
The known-answer tests restate the reference's ``tests/test_mps_model.py``
cases for each layer of the path on the oracle's functions.
"""
import numpy as np
import pytest
import torch

from fast_audiovae import weights as W
from oracle import decoder as D


def array(shape, seed=7):
    return np.random.default_rng(seed).normal(0, 0.1, shape).astype(np.float32)


@pytest.fixture(scope="module")
def oracle0():
    return D.Decoder(W.seeded_weights(0))


def test_seeded_weights_are_the_golden_ones(golden):
    import hashlib
    g = golden("decoder_seed0.npz")
    w = W.seeded_weights(0)
    h = hashlib.sha256()
    for name in W.weight_shapes():
        h.update(name.encode())
        h.update(np.ascontiguousarray(w[name], np.float32).tobytes())
    assert h.hexdigest() == str(g["weights_sha256"])
    assert np.array_equal(g["z3"], W.seeded_latents(0, 3))


def test_oracle_batch_matches_reference_decoder(golden, oracle0):
    g = golden("decoder_seed0.npz")
    torch.set_num_threads(1)
    for key in ("3", "25"):
        audio = oracle0.decode_numpy(g["z" + key])
        d = D.discrepancy(g["audio" + key], audio)
        assert d["max_abs"] <= 1e-6, d


def test_oracle_stream_matches_reference_stream(golden, oracle0):
    g = golden("decoder_seed0.npz")
    torch.set_num_threads(1)
    out = oracle0.stream_numpy(g["z25"], (1, 7, 2, 3, 11))
    assert D.discrepancy(g["stream25_uneven"], out)["max_abs"] <= 1e-6


def test_oracle_histories_match_reference(golden, oracle0):
    g = golden("decoder_seed0.npz")
    _, states = oracle0.decode(g["z3"])
    assert set(states) == set(W.state_shapes())
    for key in g:
        if key.startswith("state3/"):
            name = key[len("state3/"):]
            np.testing.assert_allclose(states[name].numpy(), g[key], atol=1e-6, rtol=0)


def test_seeded_init_does_not_saturate(golden):
    audio = golden("decoder_seed0.npz")["audio25"]
    assert 0.2 < float(audio.std()) < 0.8
    assert float(np.mean(np.abs(audio) > 0.999)) < 0.01


# --- known answers restated from the reference's tests/test_mps_model.py ------------

@pytest.mark.parametrize("dilation", [1, 3, 9])
def test_depthwise_partitions_match_python_loop(dilation):
    """``test_mps_model.py:14-37``: chunk partitions (1,0,2,3,9) equal one loop."""
    weight, bias, x = array((3, 1, 7)), array((3,), 8), array((1, 3, 15), 9)
    initial = array((1, 3, 6 * dilation), 10)
    joined = np.concatenate((initial, x), axis=-1)
    expected = np.empty_like(x)
    for c in range(3):
        for t in range(15):
            expected[0, c, t] = bias[c] + sum(float(weight[c, 0, k]) * float(joined[0, c, t + k * dilation])
                                              for k in range(7))
    state = torch.from_numpy(initial.copy())
    chunks, pos = [], 0
    for length in (1, 0, 2, 3, 9):
        y, state = D.causal_conv(torch.from_numpy(x[..., pos:pos + length].copy()), state,
                                 torch.from_numpy(weight), torch.from_numpy(bias), dilation, 3)
        chunks.append(y)
        pos += length
    np.testing.assert_allclose(torch.cat(chunks, dim=-1).numpy(), expected, atol=2e-7, rtol=2e-6)
    np.testing.assert_array_equal(state.numpy(), joined[..., -6 * dilation:])


def transpose_oracle(x, history, weight, bias, stride):
    """Float64 scatter form of the causal transposed conv (``test_mps_model.py:40-49``)."""
    joined = np.concatenate((history, x), axis=-1)
    result = np.zeros((1, weight.shape[1], (joined.shape[-1] + 1) * stride), dtype=np.float64)
    for t in range(joined.shape[-1]):
        for i in range(weight.shape[0]):
            for o in range(weight.shape[1]):
                for k in range(2 * stride):
                    result[0, o, t * stride + k] += float(joined[0, i, t]) * float(weight[i, o, k])
    result += bias[None, :, None]
    return result[..., stride:stride + x.shape[-1] * stride].astype(np.float32)


@pytest.mark.parametrize("paired", [False, True])
@pytest.mark.parametrize("stride", [2, 5, 6, 8])
@pytest.mark.parametrize("pattern", ["signed", "quiet", "zero"])
def test_transpose_matches_scatter_oracle(stride, paired, pattern):
    """``test_mps_model.py:52-94``: chunked polyphase form == float64 scatter, causal."""
    weight, bias = array((3, 2, 2 * stride)), array((2,), 11)
    x, initial = array((1, 3, 7), 12), array((1, 3, 1), 13)
    if pattern == "quiet":
        x *= np.float32(1e-5)
        initial *= np.float32(1e-5)
    elif pattern == "zero":
        x.fill(0)
        initial.fill(0)
    packed = D.pack_transpose(torch.from_numpy(weight), stride, paired)
    expected = transpose_oracle(x, initial, weight, bias, stride)
    state, chunks, pos = torch.from_numpy(initial.copy()), [], 0
    for length in (1, 0, 3, 1, 2):
        packet = torch.from_numpy(x[..., pos:pos + length].copy())
        y, state = D.causal_transpose(packet, state, packed, torch.from_numpy(bias), stride, paired)
        assert tuple(y.shape) == (1, 2, length * stride)
        chunks.append(y)
        pos += length
    actual = torch.cat(chunks, dim=-1).numpy()
    np.testing.assert_allclose(actual, expected, atol=2e-7, rtol=2e-6)
    changed = x.copy()
    changed[..., 4:] += np.float32(0.7)
    prefix, _ = D.causal_transpose(torch.from_numpy(changed), torch.from_numpy(initial.copy()), packed,
                                   torch.from_numpy(bias), stride, paired)
    np.testing.assert_allclose(prefix.numpy()[..., :4 * stride], actual[..., :4 * stride], atol=2e-7, rtol=2e-6)


@pytest.mark.parametrize("paired", [False, True])
@pytest.mark.parametrize("stride", [2, 5, 6, 8])
def test_transpose_bias_added_once(stride, paired):
    """``test_mps_model.py:97-113``: first call 9.0, second 11.0, history = input."""
    weight = np.concatenate((np.ones((1, 1, stride), np.float32), np.full((1, 1, stride), 2, np.float32)), -1)
    packed = D.pack_transpose(torch.from_numpy(weight), stride, paired)
    bias = torch.tensor([8.0])
    x = torch.ones(1, 1, 1)
    first, state = D.causal_transpose(x, torch.zeros(1, 1, 1), packed, bias, stride, paired)
    assert torch.equal(first, torch.full((1, 1, stride), 9.0)) and torch.equal(state, x)
    second, _ = D.causal_transpose(x, state, packed, bias, stride, paired)
    assert torch.equal(second, torch.full((1, 1, stride), 11.0))


@pytest.mark.parametrize("channels", [(3, 5), (5, 3)])
@pytest.mark.parametrize("length", [1, 2, 13])
def test_pointwise_matches_conv1d(channels, length):
    """``test_mps_model.py:155-164``."""
    cin, cout = channels
    weight, bias = array((cout, cin, 1), 20), array((cout,), 21)
    x = torch.from_numpy(array((1, cin, length), 22))
    ref = torch.nn.functional.conv1d(x, torch.from_numpy(weight), torch.from_numpy(bias))
    torch.testing.assert_close(D.pointwise(x, torch.from_numpy(weight), torch.from_numpy(bias)), ref,
                               atol=2e-7, rtol=2e-6)


def test_snake_uses_literal_reciprocal():
    """``test_mps_model.py:167-177``: the stored reciprocal, not 1/alpha."""
    alpha = torch.tensor([2.0, 3.0])
    reciprocal = torch.tensor([0.3, 0.1])
    x = torch.tensor([[[0., 0.2, -0.4], [0.1, -0.3, 0.5]]])
    sine = torch.sin(alpha.reshape(1, 2, 1) * x)
    assert torch.equal(D.snake(x, alpha, reciprocal), x + reciprocal.reshape(1, 2, 1) * (sine * sine))


def test_snake_dw_snake_matches_reference_c_kernel(golden):
    """Oracle Snake -> DW7 -> Snake vs the reference x86 C kernel (scalar libm sine)."""
    g = golden("elementwise.npz")
    for d in (1, 3, 9):
        p = f"sds{d}/"
        x = torch.from_numpy(g[p + "x"])
        h = D.snake(x, torch.from_numpy(g[p + "a1"]), torch.from_numpy(g[p + "r1"]))
        y, _ = D.causal_conv(h, torch.zeros(1, 8, 6 * d), torch.from_numpy(g[p + "w"][:, None, :]),
                             torch.from_numpy(g[p + "b"]), d, 8)
        y = D.snake(y, torch.from_numpy(g[p + "a2"]), torch.from_numpy(g[p + "r2"]))
        np.testing.assert_allclose(y.numpy(), g[p + "y"], atol=2e-6, rtol=2e-6)
    expected = g["br/skip"] + (g["br/product"] + g["br/bias"][None, :, None])
    assert np.array_equal(expected, g["br/y"])


def test_state_inventory_matches_reference():
    shapes = D.state_shapes()
    assert shapes == W.state_shapes()
    assert len(shapes) == 26 and sum(int(np.prod(s)) * 4 for s in shapes.values()) == 647424


def test_empty_decode_preserves_histories(oracle0):
    _, states = oracle0.decode(W.seeded_latents(3, 2))
    audio, same = oracle0.decode(np.zeros((1, 64, 0), np.float32), states)
    assert audio.shape == (1, 1, 0)
    assert all(torch.equal(states[k], same[k]) for k in states)
