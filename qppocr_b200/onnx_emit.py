"""ONNX files of the synthetic nets, so the reference's own CPU path can time
the same networks this backend runs.

The reference loads models only from ONNX bytes (`load_onnx_memory`,
crates/qppocr-core/src/onnx/parse.rs:550-749) found in a model directory
(crates/qppocr/src/models.rs:88-170: `<dir>/<tier>/det.onnx`,
`<dir>/<tier>/rec.onnx`, `<dir>/cls.onnx`), and its benchmark
(`qppocr bench`, crates/qppocr-cli/src/main.rs:741-880) reads a list of image
files.  The `onnx` package is not available here, so the protobuf wire format
is written directly:

* ModelProto: ir_version (1), producer_name (2), producer_version (3),
  graph (7), opset_import (8, domain "" = ai.onnx), metadata_props (14).
* GraphProto: node (1), name (2), initializer (5), input (11), output (12).
* NodeProto: input (1), output (2), name (3), op_type (4), attribute (5).
* AttributeProto: name (1), f (2), i (3), s (4), floats (7), ints (8),
  type (20).
* TensorProto: dims (1), data_type (2), name (8), raw_data (9), little
  endian; FLOAT weights, INT64 shape / axis constants.
* ValueInfoProto: name (1), type (2) -> tensor_type (1) -> elem_type (1),
  shape (2) -> dim (1) -> dim_value (1) or dim_param (2) for a dynamic axis.

Fields are written in field-number order and repeated scalars unpacked: the
canonical proto2 encoding of onnx.proto, as protobuf itself serialises it.

These are the fields parse.rs reads (parse.rs:148-300 tensors, :317-373
attributes, :376-408 nodes, :428-501 value infos, :503-548 graph,
:550-627 model).  The rec model carries its dictionary as the `character`
metadata entry (the converted-model path, pipeline/engine.rs:365-380), sized
so blank + entries + space equals the head's class count
(engine.rs:447-470).

    python -m qppocr_b200.onnx_emit OUT_DIR [--tier small] [--images 16] [--hw 960]

writes OUT_DIR/<tier>/det.onnx, OUT_DIR/<tier>/rec.onnx, OUT_DIR/cls.onnx and
OUT_DIR/images/img_NNNN.png (seeded RGB noise).  `qppocr bench` checks model
files against the upstream SHA-256 unless the engine is built with
`verify_sha256(false)` (crates/qppocr/src/lib.rs:521-525).
"""
from __future__ import annotations

import argparse
import os
import struct
import sys
import zlib
from typing import Dict, Iterable, List, Optional, Sequence

import numpy as np

from .graph import Graph

IR_VERSION = 8
OPSET = 17

# TensorProto.DataType
DT_FLOAT, DT_INT64 = 1, 7
# AttributeProto.AttributeType
AT_FLOAT, AT_INT, AT_STRING, AT_FLOATS, AT_INTS = 1, 2, 3, 6, 7


# ------------------------------------------------------------ wire format
def _varint(v: int) -> bytes:
    if v < 0:
        v += 1 << 64  # int64 fields: two's complement, ten bytes
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wire: int) -> bytes:
    return _varint((field << 3) | wire)


def _len_field(field: int, payload: bytes) -> bytes:
    return _key(field, 2) + _varint(len(payload)) + payload


def _str_field(field: int, s: str) -> bytes:
    return _len_field(field, s.encode("utf-8"))


def _int_field(field: int, v: int) -> bytes:
    return _key(field, 0) + _varint(int(v))


def _f32_field(field: int, v: float) -> bytes:
    return _key(field, 5) + struct.pack("<f", np.float32(v))


# ------------------------------------------------------------ messages
def tensor_proto(name: str, arr: np.ndarray) -> bytes:
    """TensorProto with raw little-endian data: float32 -> FLOAT, integer -> INT64."""
    a = np.asarray(arr)
    if a.dtype.kind == "f":
        dt, raw = DT_FLOAT, np.ascontiguousarray(a, "<f4").tobytes()
    elif a.dtype.kind in "iub":
        dt, raw = DT_INT64, np.ascontiguousarray(a, "<i8").tobytes()
    else:
        raise TypeError(f"{name}: unsupported weight dtype {a.dtype}")
    out = b"".join(_int_field(1, int(d)) for d in a.shape)
    out += _int_field(2, dt)
    out += _str_field(8, name)
    out += _len_field(9, raw)
    return out


def attribute_proto(name: str, v) -> bytes:
    out = _str_field(1, name)
    if isinstance(v, bool) or isinstance(v, (int, np.integer)):
        return out + _int_field(3, int(v)) + _int_field(20, AT_INT)
    if isinstance(v, (float, np.floating)):
        return out + _f32_field(2, float(v)) + _int_field(20, AT_FLOAT)
    if isinstance(v, str):
        return out + _str_field(4, v) + _int_field(20, AT_STRING)
    if isinstance(v, (list, tuple)):
        if all(isinstance(e, (int, np.integer)) and not isinstance(e, bool) for e in v):
            return out + b"".join(_int_field(8, int(e)) for e in v) + _int_field(20, AT_INTS)
        if all(isinstance(e, (float, np.floating, int, np.integer)) for e in v):
            return out + b"".join(_f32_field(7, e) for e in v) + _int_field(20, AT_FLOATS)
    raise TypeError(f"attribute {name}: unsupported value {v!r}")


def node_proto(n) -> bytes:
    out = b"".join(_str_field(1, i) for i in n.inputs)
    out += b"".join(_str_field(2, o) for o in n.outputs)
    out += _str_field(3, n.name)
    out += _str_field(4, n.op_type)
    out += b"".join(_len_field(5, attribute_proto(k, v)) for k, v in n.attrs.items())
    return out


def value_info_proto(name: str, dims: Optional[Sequence[int]] = None, elem_type: int = DT_FLOAT) -> bytes:
    """A float tensor's ValueInfoProto; a 0 in `dims` is written as a named
    dynamic axis (dim_param), which the reference reads back as 0."""
    tt = _int_field(1, elem_type)
    if dims is not None:
        shape = b""
        for k, d in enumerate(dims):
            dim = _int_field(1, int(d)) if d > 0 else _str_field(2, f"{name}_dim{k}")
            shape += _len_field(1, dim)
        tt += _len_field(2, shape)
    return _str_field(1, name) + _len_field(2, _len_field(1, tt))


def graph_proto(g: Graph, w: Dict[str, np.ndarray], name: str) -> bytes:
    used = {i for n in g.nodes for i in n.inputs if i}
    out = b"".join(_len_field(1, node_proto(n)) for n in g.nodes)
    out += _str_field(2, name)
    out += b"".join(_len_field(5, tensor_proto(k, w[k])) for k in w if k in used)
    dims = list(g.input_dims) + [None] * (len(g.inputs) - len(g.input_dims))
    out += b"".join(_len_field(11, value_info_proto(i, d)) for i, d in zip(g.inputs, dims))
    out += b"".join(_len_field(12, value_info_proto(o)) for o in g.outputs)
    return out


def model_bytes(g: Graph, w: Dict[str, np.ndarray], name: str = "graph",
                metadata: Optional[Dict[str, str]] = None) -> bytes:
    """Serialise one graph and its weights as an ONNX ModelProto."""
    out = _int_field(1, IR_VERSION)
    out += _str_field(2, "qppocr_b200.nets")
    out += _str_field(3, "1")
    out += _len_field(7, graph_proto(g, w, name))
    out += _len_field(8, _str_field(1, "") + _int_field(2, OPSET))
    for k, v in (metadata or {}).items():
        out += _len_field(14, _str_field(1, k) + _str_field(2, v))
    return out


def synthetic_dictionary(n_entries: int) -> str:
    """n_entries distinct one-character lines, consecutive code points from
    U+4E00 (CJK unified ideographs) skipping surrogates, newline-separated."""
    chars = []
    cp = 0x4E00
    while len(chars) < n_entries:
        if not (0xD800 <= cp <= 0xDFFF):
            chars.append(chr(cp))
        cp += 1
    return "\n".join(chars)


# ------------------------------------------------------------ images
def png_bytes(img: np.ndarray) -> bytes:
    """8-bit RGB PNG (no filtering, one IDAT) of an [h, w, 3] uint8 array."""
    img = np.ascontiguousarray(img, np.uint8)
    h, w, c = img.shape
    assert c == 3

    def chunk(tag: bytes, data: bytes) -> bytes:
        return struct.pack(">I", len(data)) + tag + data + struct.pack(">I", zlib.crc32(tag + data) & 0xFFFFFFFF)

    rows = np.concatenate([np.zeros((h, 1), np.uint8), img.reshape(h, w * 3)], axis=1)
    return (b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", struct.pack(">IIBBBBB", w, h, 8, 2, 0, 0, 0))
            + chunk(b"IDAT", zlib.compress(rows.tobytes(), 6)) + chunk(b"IEND", b""))


def synthetic_images(n: int, h: int, w: int, seed: int = 7) -> Iterable[np.ndarray]:
    rng = np.random.Generator(np.random.PCG64(seed))
    for _ in range(n):
        yield rng.integers(0, 256, (h, w, 3), dtype=np.uint8)


# ------------------------------------------------------------ model directory
def write_model_dir(root: str, tier: str = "small", n_images: int = 16, hw: int = 960) -> List[str]:
    """The reference's model-directory layout for the synthetic det / rec /
    cls nets, plus n_images seeded PNGs; returns the paths written."""
    from . import nets

    written = []
    os.makedirs(os.path.join(root, tier), exist_ok=True)
    g, w = nets.build_det()
    written.append(_write(os.path.join(root, tier, "det.onnx"), model_bytes(g, w, "det")))
    g, w = nets.build_rec()
    classes = w[[n for n in g.nodes if n.op_type == "MatMul"][-1].inputs[1]].shape[1]
    meta = {"character": synthetic_dictionary(classes - 2)}  # blank + entries + space
    written.append(_write(os.path.join(root, tier, "rec.onnx"), model_bytes(g, w, "rec", meta)))
    g, w = nets.build_cls()
    written.append(_write(os.path.join(root, "cls.onnx"), model_bytes(g, w, "cls")))
    os.makedirs(os.path.join(root, "images"), exist_ok=True)
    for k, img in enumerate(synthetic_images(n_images, hw, hw)):
        written.append(_write(os.path.join(root, "images", f"img_{k:04d}.png"), png_bytes(img)))
    return written


def _write(path: str, data: bytes) -> str:
    with open(path, "wb") as f:
        f.write(data)
    return path


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m qppocr_b200.onnx_emit")
    ap.add_argument("out_dir")
    ap.add_argument("--tier", default="small", choices=["tiny", "small", "medium"])
    ap.add_argument("--images", type=int, default=16)
    ap.add_argument("--hw", type=int, default=960)
    a = ap.parse_args(argv)
    for p in write_model_dir(a.out_dir, a.tier, a.images, a.hw):
        print(p, os.path.getsize(p))
    return 0


if __name__ == "__main__":
    sys.exit(main())
