"""Writes a small AudioVAE2-decoder-shaped ONNX model for the importer tests.

No ``onnx`` package is available here, so this encodes the protobuf wire
format directly. The graph follows the structure the reference's
``MPSModel.from_onnx`` reads (``src/fast_audiovae/mps_decoder.py:190-286``):
convolution weights named ``audio_vae.decoder.model.<k>[.block.<j>...]``, the
stage affine constants ``unsqueeze`` / ``unsqueeze_<n>`` of shape [1, C, 1],
and each Snake as ``Mul(x, alpha) -> Sin -> Pow(., 2) -> Mul(., reciprocal) ->
Add(x, .)`` (``graph/elementwise.py:117-165``). It is not a runnable decoder
export (no causal crops); it carries the coefficients in every storage form
the importer handles: inline raw bytes, typed float lists, Constant nodes and
external data (tensors of 1 KiB and more go to ``<name>.data``, as the pinned
export keeps its weights).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

ROOT = "audio_vae.decoder.model."
RATES = (8, 6, 5, 2, 2, 2)
DILATIONS = (1, 3, 9)


def _varint(v):
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field, wire):
    return _varint((field << 3) | wire)


def _int(field, v):
    return _key(field, 0) + _varint(v)


def _bytes(field, payload):
    return _key(field, 2) + _varint(len(payload)) + payload


def _str(field, s):
    return _bytes(field, s.encode())


def _packed(field, values):
    return _bytes(field, b"".join(_varint(v) for v in values))


class ExternalData:
    def __init__(self, name):
        self.name = name
        self.blob = bytearray()

    def add(self, raw):
        offset = len(self.blob)
        self.blob += raw
        pad = (-len(self.blob)) % 64
        self.blob += b"\0" * pad
        return offset


def tensor(name, array, external=None, typed=False):
    a = np.ascontiguousarray(array, dtype=np.float32)
    out = _packed(1, list(a.shape)) + _int(2, 1) + _str(8, name)
    raw = a.astype("<f4").tobytes()
    if external is not None and len(raw) >= 1024:
        offset = external.add(raw)
        for k, v in (("location", external.name), ("offset", str(offset)), ("length", str(len(raw)))):
            out += _bytes(13, _str(1, k) + _str(2, v))
        out += _int(14, 1)
    elif typed:
        out += _bytes(4, raw)  # packed float_data
    else:
        out += _bytes(9, raw)
    return out


def attr_int(name, v):
    return _str(1, name) + _int(20, 2) + _int(3, v)


def attr_ints(name, values):
    return _str(1, name) + _int(20, 7) + _packed(8, values)


def attr_str(name, value):
    return _str(1, name) + _int(20, 3) + _bytes(4, value)


def attr_tensor(name, payload):
    return _str(1, name) + _int(20, 4) + _bytes(5, payload)


def node(op, inputs, outputs, name, attrs=()):
    out = b"".join(_str(1, i) for i in inputs) + b"".join(_str(2, o) for o in outputs)
    out += _str(3, name) + _str(4, op)
    return out + b"".join(_bytes(5, a) for a in attrs)


def value_info(name, dims):
    shape = b"".join(_bytes(1, _int(1, d) if isinstance(d, int) else _str(2, d)) for d in dims)
    return _str(1, name) + _bytes(2, _bytes(1, _int(1, 1) + _bytes(2, shape)))


class _Builder:
    def __init__(self, external):
        self.nodes, self.inits, self.infos = [], [], []
        self.external = external
        self.count = 0
        self.snakes = 0

    def fresh(self, hint):
        self.count += 1
        return f"{hint}_{self.count}"

    def init(self, name, array, typed=False):
        self.inits.append(tensor(name, array, self.external, typed))

    def conv(self, x, name, w, b, *, dilation=1, groups=1, transpose=False, stride=1):
        self.init(name + ".weight", w)
        self.init(name + ".bias", b, typed=True)
        pads = [0, 0] if transpose or w.shape[2] == 1 else [6 * dilation, 0]
        attrs = [attr_int("group", groups), attr_ints("pads", pads), attr_str("auto_pad", b"NOTSET"),
                 attr_ints("strides", [stride]), attr_ints("dilations", [dilation])]
        if transpose:
            attrs.append(attr_ints("output_padding", [0]))
        y = self.fresh("conv")
        self.nodes.append(node("ConvTranspose" if transpose else "Conv", [x, name + ".weight", name + ".bias"], [y],
                               self.fresh("node"), attrs))
        return y

    def snake(self, x, alpha, recip):
        c = alpha.size
        k = self.snakes
        self.snakes += 1
        self.infos.append(value_info(x, [1, c, "T"]))
        a_name, r_name = f"snake{k}.alpha", f"snake{k}.reciprocal"
        self.init(a_name, alpha.reshape(1, c, 1))
        if k % 2:  # every other reciprocal as a Constant node, shape [C, 1]
            self.nodes.append(node("Constant", [], [r_name], self.fresh("node"),
                                   [attr_tensor("value", tensor(r_name, recip.reshape(c, 1)))]))
        else:
            self.init(r_name, recip.reshape(1, c, 1))
        m, s, q, corr, y = (self.fresh(h) for h in ("mul", "sin", "sq", "corr", "snake"))
        self.nodes.append(node("Mul", [x, a_name] if k % 3 else [a_name, x], [m], self.fresh("node")))
        self.nodes.append(node("Sin", [m], [s], self.fresh("node")))
        if k % 2:
            self.nodes.append(node("Mul", [s, s], [q], self.fresh("node")))
        else:
            self.nodes.append(node("Pow", [s, "two"], [q], self.fresh("node")))
        self.nodes.append(node("Mul", [q, r_name], [corr], self.fresh("node")))
        self.nodes.append(node("Add", [x, corr], [y], self.fresh("node")))
        return y


def write_decoder(directory, w, name="audio_vae_decoder.onnx", mutate=None):
    """Writes ``name`` and ``name + '.data'`` into ``directory`` from coefficient
    dict ``w`` (this package's names); returns the model path. ``mutate`` may
    edit the node list before encoding (for negative tests)."""
    directory = Path(directory)
    external = ExternalData(name + ".data")
    b = _Builder(external)
    b.init("two", np.array(2.0, np.float32))
    x = b.conv("z", ROOT + "0", w["stem.weight"], w["stem.bias"], groups=64)
    x = b.conv(x, ROOT + "1", w["pointwise.weight"], w["pointwise.bias"])
    channels = 2048
    for i, s in enumerate(RATES):
        p, prefix, cout = f"stage{i}.", ROOT + str(i + 2) + ".block.", channels // 2
        scale_name = "unsqueeze" if i == 0 else f"unsqueeze_{2 * i}"
        b.init(scale_name, w[p + "scale"].reshape(1, channels, 1))
        b.init(f"unsqueeze_{2 * i + 1}", w[p + "offset"].reshape(1, channels, 1))
        a, c = b.fresh("scaled"), b.fresh("shifted")
        b.nodes.append(node("Mul", [x, scale_name], [a], b.fresh("node")))
        b.nodes.append(node("Add", [a, f"unsqueeze_{2 * i + 1}"], [c], b.fresh("node")))
        x = b.snake(c, w[p + "snake.alpha"], w[p + "snake.reciprocal"])
        x = b.conv(x, prefix + "1", w[p + "transpose.weight"], w[p + "transpose.bias"], transpose=True, stride=s)
        for j, d in enumerate(DILATIONS):
            r, unit = f"{p}residual{j}.", prefix + str(j + 2) + ".block."
            h = b.snake(x, w[r + "pre.alpha"], w[r + "pre.reciprocal"])
            h = b.conv(h, unit + "1", w[r + "depthwise.weight"], w[r + "depthwise.bias"], dilation=d, groups=cout)
            h = b.snake(h, w[r + "post.alpha"], w[r + "post.reciprocal"])
            h = b.conv(h, unit + "3", w[r + "pointwise.weight"], w[r + "pointwise.bias"])
            y = b.fresh("residual")
            b.nodes.append(node("Add", [x, h], [y], b.fresh("node")))
            x = y
        channels = cout
    x = b.snake(x, w["final.snake.alpha"], w["final.snake.reciprocal"])
    x = b.conv(x, ROOT + "9", w["final.weight"], w["final.bias"])
    b.nodes.append(node("Tanh", [x], ["audio"], b.fresh("node")))
    nodes = b.nodes if mutate is None else mutate(list(b.nodes))
    graph = b"".join(_bytes(1, n) for n in nodes) + _str(2, "audio_vae_decoder")
    graph += b"".join(_bytes(5, t) for t in b.inits)
    graph += _bytes(11, value_info("z", [1, 64, "L"])) + _bytes(12, value_info("audio", [1, 1, "S"]))
    graph += b"".join(_bytes(13, v) for v in b.infos)
    model = _int(1, 8) + _bytes(8, _str(1, "") + _int(2, 17)) + _str(2, "fast-audiovae-tests") + _bytes(7, graph)
    path = directory / name
    path.write_bytes(model)
    (directory / external.name).write_bytes(bytes(external.blob))
    return path
