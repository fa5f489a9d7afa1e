"""Coefficient import from an AudioVAE2 ONNX export (CPU).

The reference builds its decoder from the pinned export's initializers
(``src/fast_audiovae/mps_decoder.py:190-286``). The pinned files are not in
this container, so a decoder-shaped model with the reference's tensor names,
convolution attributes and Snake patterns is written by ``tests/onnx_writer.py``
from known coefficients; the importer must give those coefficients back bit
for bit, and reject a changed graph.
"""
import numpy as np
import pytest

import onnx_writer
from fast_audiovae import onnx_import
from fast_audiovae import weights as W


@pytest.fixture(scope="module")
def coefficients():
    return W.seeded_weights(7)


def test_import_returns_the_written_coefficients(tmp_path, coefficients):
    path = onnx_writer.write_decoder(tmp_path, coefficients)
    assert (tmp_path / "audio_vae_decoder.onnx.data").stat().st_size > 50_000_000  # weights stored externally
    got = onnx_import.load_coefficients(path, pinned=False)
    assert list(got) == list(W.weight_shapes())
    for name, value in coefficients.items():
        assert got[name].dtype == np.float32 and got[name].shape == value.shape, name
        assert np.array_equal(got[name].view(np.uint32), value.view(np.uint32)), name


def test_pinned_mode_requires_the_pinned_files(tmp_path, coefficients):
    path = onnx_writer.write_decoder(tmp_path, coefficients)
    with pytest.raises(onnx_import.OnnxFormatError, match="pinned"):
        onnx_import.load_coefficients(path)


def test_changed_attributes_are_rejected(tmp_path, coefficients):
    """The stage-0 unit-0 depthwise conv (dilation 1) claiming dilation 3."""
    good = onnx_writer._bytes(5, onnx_writer.attr_ints("dilations", [1]))
    bad = onnx_writer._bytes(5, onnx_writer.attr_ints("dilations", [3]))
    key = onnx_writer._str(1, onnx_writer.ROOT + "2.block.2.block.1.weight")

    def mutate(nodes):
        i = next(k for k, n in enumerate(nodes) if key in n)
        nodes[i] = nodes[i].replace(good, bad)
        return nodes

    path = onnx_writer.write_decoder(tmp_path, coefficients, mutate=mutate)
    with pytest.raises(onnx_import.OnnxFormatError, match="attributes changed"):
        onnx_import.load_coefficients(path, pinned=False)


def test_missing_snake_is_rejected(tmp_path, coefficients):
    def mutate(nodes):
        sins = [k for k, n in enumerate(nodes) if onnx_writer._str(4, "Sin") in n]
        del nodes[sins[5]]
        return nodes

    path = onnx_writer.write_decoder(tmp_path, coefficients, mutate=mutate)
    with pytest.raises(onnx_import.OnnxFormatError):
        onnx_import.load_coefficients(path, pinned=False)


def test_facade_reads_onnx_sources(tmp_path, coefficients):
    import fast_audiovae
    path = onnx_writer.write_decoder(tmp_path, coefficients)
    got, origin = fast_audiovae._coefficients(None, str(path), 0, pinned=False)
    assert origin.startswith("onnx:")
    assert all(np.array_equal(got[k], v) for k, v in coefficients.items())
