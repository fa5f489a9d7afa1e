"""Decoder coefficients from the AudioVAE2 ONNX export, without the ``onnx`` package.

The reference loads the checksum-pinned export (``src/fast_audiovae/assets.py:6-11``:
``audio_vae_decoder.onnx`` plus its external-data file) and assembles its fp32
decoder from the graph's initializers in ``MPSModel.from_onnx``
(``src/fast_audiovae/mps_decoder.py:190-286``):

* convolution weights and biases by name (``audio_vae.decoder.model.<k>...``),
  each checked against its consumer node's attributes (group, causal pads,
  strides, dilations);
* the per-stage affine ``unsqueeze`` / ``unsqueeze_<n>`` constants, shape
  ``[1, C, 1]``;
* the 43 Snake coefficient pairs by matching ``Mul(x, alpha) -> Sin -> square
  -> Mul(., reciprocal) -> Add(x, .)`` in graph order
  (``graph/elementwise.py:117-165``), consumed stage by stage (stage Snake, then
  per residual unit pre and post) and finally the output Snake.

This module restates that mapping over a minimal reader of the protobuf wire
format (the ONNX ``ModelProto`` / ``GraphProto`` / ``NodeProto`` /
``TensorProto`` fields it needs, including external data), and returns the 188
coefficient arrays under this package's names (``weights.weight_shapes()``).
With ``pinned=True`` (the reference's only mode) the files must carry the
pinned SHA-256 digests, and the graph the pinned contract's totals (402 nodes,
216 initializers).
"""
from __future__ import annotations

import hashlib
import struct
from pathlib import Path

import numpy as np

from . import weights as W

# The reference's pins (src/fast_audiovae/assets.py:8-11).
PINNED_FILES = {
    "audio_vae_decoder.onnx": "fdd20e200675ab9649bf33f16bc5974101ba5cf47ab89fbfe29f3d36ff6c3c84",
    "audio_vae_decoder.onnx.data": "3b76bd57356e96893655bd24a364989e016c5af2fc8c29195caaefb4eccf5143",
}
ROOT = "audio_vae.decoder.model."

# TensorProto.DataType values used here.
_FLOAT, _INT32, _INT64, _DOUBLE = 1, 6, 7, 11
_NUMPY = {_FLOAT: np.float32, _INT32: np.int32, _INT64: np.int64, _DOUBLE: np.float64}


class OnnxFormatError(ValueError):
    """The file is not an ONNX model this reader understands, or its graph
    differs from the AudioVAE2 decoder contract."""


def _require(condition, message):
    if not condition:
        raise OnnxFormatError(message)


# ------------------------------------------------------------- wire format
def _varint(buf, pos):
    result = shift = 0
    while True:
        _require(pos < len(buf), "truncated varint")
        b = buf[pos]
        pos += 1
        result |= (b & 0x7F) << shift
        if b < 0x80:
            return result, pos
        shift += 7
        _require(shift < 70, "varint too long")


def _fields(buf):
    """(field number, wire type, value) of a message: ints for varint and fixed
    fields, memoryviews for length-delimited ones."""
    pos, end = 0, len(buf)
    while pos < end:
        key, pos = _varint(buf, pos)
        field, wire = key >> 3, key & 7
        if wire == 0:
            value, pos = _varint(buf, pos)
        elif wire == 1:
            _require(pos + 8 <= end, "truncated fixed64")
            value = struct.unpack_from("<Q", buf, pos)[0]
            pos += 8
        elif wire == 2:
            n, pos = _varint(buf, pos)
            _require(pos + n <= end, "truncated field")
            value = buf[pos:pos + n]
            pos += n
        elif wire == 5:
            _require(pos + 4 <= end, "truncated fixed32")
            value = struct.unpack_from("<I", buf, pos)[0]
            pos += 4
        else:
            raise OnnxFormatError(f"unsupported wire type {wire}")
        yield field, wire, value


def _signed(v):
    return v - (1 << 64) if v >= 1 << 63 else v


def _ints(wire, value):
    """A repeated int64 field element: one varint, or a packed run."""
    if wire == 0:
        return [_signed(value)]
    out, pos = [], 0
    while pos < len(value):
        v, pos = _varint(value, pos)
        out.append(_signed(v))
    return out


def _text(value):
    return bytes(value).decode("utf-8")


class Tensor:
    """A TensorProto: name, dims, data type and its bytes (inline or external)."""

    def __init__(self, buf):
        self.name, self.dims, self.dtype = "", [], 0
        self.raw = None
        self.floats, self.int64s, self.int32s, self.doubles = [], [], [], []
        self.external = {}
        self.location = 0
        for f, w, v in _fields(buf):
            if f == 1:
                self.dims += _ints(w, v)
            elif f == 2:
                self.dtype = v
            elif f == 4:
                self.floats += (list(struct.unpack(f"<{len(v) // 4}f", v)) if w == 2
                                else [struct.unpack("<f", struct.pack("<I", v))[0]])
            elif f == 5:
                self.int32s += _ints(w, v)
            elif f == 7:
                self.int64s += _ints(w, v)
            elif f == 8:
                self.name = _text(v)
            elif f == 9:
                self.raw = bytes(v)
            elif f == 10:
                self.doubles += (list(struct.unpack(f"<{len(v) // 8}d", v)) if w == 2
                                 else [struct.unpack("<d", struct.pack("<Q", v))[0]])
            elif f == 13:
                entry = dict((k, _text(x)) for k, _, x in _fields(v))
                self.external[entry.get(1, "")] = entry.get(2, "")
            elif f == 14:
                self.location = v

    def array(self, base_dir):
        _require(self.dtype in _NUMPY, f"{self.name}: unsupported tensor type {self.dtype}")
        dtype = np.dtype(_NUMPY[self.dtype]).newbyteorder("<")
        count = int(np.prod(self.dims)) if self.dims else 1
        if self.location == 1:  # external data: location, offset, length (tensor.proto)
            path = Path(base_dir) / self.external.get("location", "")
            _require(path.is_file(), f"{self.name}: external data file {path} is missing")
            offset = int(self.external.get("offset", 0))
            length = int(self.external.get("length", count * dtype.itemsize))
            _require(length == count * dtype.itemsize, f"{self.name}: external length mismatch")
            with open(path, "rb") as f:
                f.seek(offset)
                data = f.read(length)
            _require(len(data) == length, f"{self.name}: external data truncated")
            a = np.frombuffer(data, dtype=dtype)
        elif self.raw is not None:
            _require(len(self.raw) == count * dtype.itemsize, f"{self.name}: raw data size mismatch")
            a = np.frombuffer(self.raw, dtype=dtype)
        else:
            vals = {_FLOAT: self.floats, _DOUBLE: self.doubles, _INT64: self.int64s, _INT32: self.int32s}[self.dtype]
            _require(len(vals) == count, f"{self.name}: typed data size mismatch")
            a = np.asarray(vals, dtype=dtype)
        return np.array(a.reshape(self.dims), dtype=dtype.newbyteorder("="), copy=True)


class Node:
    """A NodeProto: op type, domain, inputs, outputs and attributes."""

    def __init__(self, buf):
        self.inputs, self.outputs, self.name, self.op_type, self.domain = [], [], "", "", ""
        self.attrs = {}
        for f, _, v in _fields(buf):
            if f == 1:
                self.inputs.append(_text(v))
            elif f == 2:
                self.outputs.append(_text(v))
            elif f == 3:
                self.name = _text(v)
            elif f == 4:
                self.op_type = _text(v)
            elif f == 7:
                self.domain = _text(v)
            elif f == 5:
                name, value = _attribute(v)
                self.attrs[name] = value


def _attribute(buf):
    """(name, value) of an AttributeProto: int, float, bytes, tensor or int list."""
    name, value, ints, floats = "", None, [], []
    for f, w, v in _fields(buf):
        if f == 1:
            name = _text(v)
        elif f == 2:
            value = struct.unpack("<f", struct.pack("<I", v))[0]
        elif f == 3:
            value = _signed(v)
        elif f == 4:
            value = bytes(v)
        elif f == 5:
            value = Tensor(v)
        elif f == 7:
            floats += (list(struct.unpack(f"<{len(v) // 4}f", v)) if w == 2
                       else [struct.unpack("<f", struct.pack("<I", v))[0]])
        elif f == 8:
            ints += _ints(w, v)
    if value is None and ints:
        value = ints
    elif value is None and floats:
        value = floats
    return name, value


def _shape(buf):
    """Dims of a ValueInfoProto's tensor type (ints, or None where symbolic)."""
    dims = None
    for f, _, v in _fields(buf):
        if f != 2:
            continue
        for tf, _, tv in _fields(v):
            if tf != 1:
                continue
            for ttf, _, ttv in _fields(tv):
                if ttf != 2:
                    continue
                dims = []
                for df, _, dv in _fields(ttv):
                    if df == 1:
                        value = None
                        for xf, _, xv in _fields(dv):
                            if xf == 1:
                                value = _signed(xv)
                        dims.append(value)
    return dims


class Graph:
    """The parts of an ONNX GraphProto the decoder mapping reads."""

    def __init__(self, path):
        path = Path(path)
        data = memoryview(path.read_bytes())
        graph = None
        for f, _, v in _fields(data):
            if f == 7:
                graph = v
        _require(graph is not None, f"{path}: no graph in the model")
        self.base_dir = path.parent
        self.nodes, self.initializers, self.inputs, self.outputs, self.shapes = [], {}, [], [], {}
        for f, _, v in _fields(graph):
            if f == 1:
                self.nodes.append(Node(v))
            elif f == 5:
                t = Tensor(v)
                self.initializers[t.name] = t
            elif f in (11, 12, 13):
                name = ""
                for vf, _, vv in _fields(v):
                    if vf == 1:
                        name = _text(vv)
                (self.inputs if f == 11 else self.outputs if f == 12 else []).append(name)
                self.shapes[name] = _shape(v)
        self.producer = {o: i for i, n in enumerate(self.nodes) for o in n.outputs}
        self.users = {}
        for i, n in enumerate(self.nodes):
            for name in set(n.inputs):
                self.users.setdefault(name, []).append(i)
        self._cache = {}

    def constant(self, name):
        """An initializer or a Constant node's value (graph inputs are not constants)."""
        if name in self.inputs:
            return None
        if name not in self._cache:
            tensor = self.initializers.get(name)
            if tensor is None:
                i = self.producer.get(name)
                node = None if i is None else self.nodes[i]
                if node is None or node.domain or node.op_type != "Constant" or not isinstance(
                        node.attrs.get("value"), Tensor):
                    return None
                tensor = node.attrs["value"]
            self._cache[name] = tensor.array(self.base_dir)
        return self._cache[name]

    def channel_constant(self, name, channels=None):
        """A per-channel constant broadcast over [1, C, T]: shape [1, C, 1] or [C, 1]
        (a scalar, or ``channels`` copies of it when given); None otherwise."""
        a = self.constant(name)
        if a is None or a.dtype != np.float32 or not np.isfinite(a).all():
            return None
        if a.ndim == 3 and a.shape[0] == 1 and a.shape[2] == 1:
            c = a.shape[1]
        elif a.ndim == 2 and a.shape[1] == 1:
            c = a.shape[0]
        elif a.size == 1 and channels:
            return np.full((channels,), a.reshape(-1)[0], dtype=np.float32)
        else:
            return None
        if channels is not None and c != channels:
            return None
        return np.array(a.reshape(c), dtype=np.float32)

    def only_user(self, name, op_type=None):
        users = self.users.get(name, [])
        if name in self.outputs or len(users) != 1:
            return None
        n = self.nodes[users[0]]
        return users[0] if not n.domain and (op_type is None or n.op_type == op_type) else None

    def snakes(self):
        """The Snake patterns in graph order: (channels, alpha, reciprocal)."""
        found = []
        for si, sin in enumerate(self.nodes):
            if sin.domain or sin.op_type != "Sin" or len(sin.inputs) != 1:
                continue
            mi = self.producer.get(sin.inputs[0])
            _require(mi is not None, "Sin without a producer")
            mul = self.nodes[mi]
            _require(mul.op_type == "Mul" and len(mul.inputs) == 2 and self.only_user(mul.outputs[0], "Sin") == si,
                     "Snake: Sin must consume a Mul(x, alpha) of its own")
            candidates = []
            for const, x in (mul.inputs, mul.inputs[::-1]):
                shape = self.shapes.get(x)
                channels = shape[1] if shape and len(shape) == 3 and isinstance(shape[1], int) else None
                alpha = self.channel_constant(const, channels)
                if alpha is not None and self.constant(x) is None:
                    candidates.append((x, alpha))
            _require(len(candidates) == 1, "Snake: alpha is not a unique per-channel constant")
            x, alpha = candidates[0]
            qi = self.only_user(sin.outputs[0])
            _require(qi is not None, "Snake: the sine must have one user")
            sq = self.nodes[qi]
            if sq.op_type == "Pow":
                e = self.constant(sq.inputs[1])
                _require(sq.inputs[0] == sin.outputs[0] and e is not None and e.size == 1
                         and float(e.reshape(-1)[0]) == 2.0, "Snake: Pow must square the sine")
            else:
                _require(sq.op_type == "Mul" and sq.inputs == [sin.outputs[0], sin.outputs[0]],
                         "Snake: the sine must be squared")
            ci = self.only_user(sq.outputs[0], "Mul")
            _require(ci is not None, "Snake: the square must feed one Mul")
            corr = self.nodes[ci]
            other = [v for v in corr.inputs if v != sq.outputs[0]]
            _require(len(other) == 1, "Snake: correction Mul")
            recip = self.channel_constant(other[0], alpha.size)
            _require(recip is not None, "Snake: reciprocal is not a per-channel constant")
            ai = self.only_user(corr.outputs[0], "Add")
            _require(ai is not None and sorted(self.nodes[ai].inputs) == sorted([x, corr.outputs[0]]),
                     "Snake: the correction must be added to x")
            found.append((alpha.size, alpha, recip))
        return found


def _sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def load_coefficients(path, *, pinned=True):
    """The 188 decoder coefficients (this package's names) from an AudioVAE2
    decoder export at ``path`` (``mps_decoder.py:190-286``)."""
    path = Path(path)
    if pinned:
        for file, digest in ((path, PINNED_FILES["audio_vae_decoder.onnx"]),
                             (path.parent / "audio_vae_decoder.onnx.data",
                              PINNED_FILES["audio_vae_decoder.onnx.data"])):
            _require(file.is_file() and _sha256(file) == digest,
                     f"This recipe requires the pinned AudioVAE2 export: {file}")
    g = Graph(path)
    if pinned:
        _require(len(g.nodes) == 402 and len(g.initializers) == 216 and g.inputs == ["z"]
                 and g.outputs == ["audio"], "Original decoder graph contract changed")
    _require(sum(n.op_type == "Conv" for n in g.nodes) == 39
             and sum(n.op_type == "ConvTranspose" for n in g.nodes) == 6, "Convolution inventory changed")
    snakes = g.snakes()
    _require(len(snakes) == 43, f"Snake inventory changed ({len(snakes)} patterns)")

    def coefficient(name, shape):
        v = g.constant(name)
        _require(v is not None and v.dtype == np.float32 and v.shape == tuple(shape) and np.isfinite(v).all(),
                 "Coefficient shape/type changed: " + name)
        return v

    def conv(name, shape, *, dilation=1, groups=1, transpose=False, stride=1):
        users = [n for n in g.nodes if len(n.inputs) == 3 and n.inputs[1] == name + ".weight"]
        _require(len(users) == 1, "Expected exactly one weight consumer: " + name)
        node = users[0]
        causal = [0, 0] if transpose or shape[2] == 1 else [6 * dilation, 0]
        want = {"group": groups, "pads": causal, "auto_pad": b"NOTSET", "strides": [stride], "dilations": [dilation]}
        if transpose:
            want["output_padding"] = [0]
        got = {k: node.attrs.get(k) for k in node.attrs if k != "kernel_shape"}
        _require(node.op_type == ("ConvTranspose" if transpose else "Conv") and got == want
                 and node.inputs[2] == name + ".bias", "Original convolution attributes changed: " + name)
        return (coefficient(name + ".weight", shape),
                coefficient(name + ".bias", (shape[1] if transpose else shape[0],)))

    order = iter(snakes)

    def snake(channels):
        c, alpha, recip = next(order)
        _require(c == channels, "Snake channel order changed")
        return alpha, recip

    out = {}
    out["stem.weight"], out["stem.bias"] = conv(ROOT + "0", (64, 1, 7), groups=64)
    out["pointwise.weight"], out["pointwise.bias"] = conv(ROOT + "1", (2048, 64, 1))
    channels = 2048
    for i, stride in enumerate(W.RATES):
        p, prefix, cout = f"stage{i}.", ROOT + str(i + 2) + ".block.", channels // 2
        out[p + "scale"] = coefficient("unsqueeze" if i == 0 else f"unsqueeze_{2 * i}", (1, channels, 1)).reshape(-1)
        out[p + "offset"] = coefficient(f"unsqueeze_{2 * i + 1}", (1, channels, 1)).reshape(-1)
        out[p + "snake.alpha"], out[p + "snake.reciprocal"] = snake(channels)
        out[p + "transpose.weight"], out[p + "transpose.bias"] = conv(
            prefix + "1", (channels, cout, 2 * stride), transpose=True, stride=stride)
        for j, d in enumerate(W.DILATIONS):
            r, unit = f"{p}residual{j}.", prefix + str(j + 2) + ".block."
            out[r + "pre.alpha"], out[r + "pre.reciprocal"] = snake(cout)
            out[r + "depthwise.weight"], out[r + "depthwise.bias"] = conv(unit + "1", (cout, 1, 7), dilation=d,
                                                                          groups=cout)
            out[r + "post.alpha"], out[r + "post.reciprocal"] = snake(cout)
            out[r + "pointwise.weight"], out[r + "pointwise.bias"] = conv(unit + "3", (cout, cout, 1))
        channels = cout
    out["final.snake.alpha"], out["final.snake.reciprocal"] = snake(32)
    out["final.weight"], out["final.bias"] = conv(ROOT + "9", (1, 32, 7))
    _require(next(order, None) is None, "Not all Snake coefficients were consumed")
    out = {k: np.ascontiguousarray(v, dtype=np.float32) for k, v in out.items()}
    W.validate_weights(out)
    return out
