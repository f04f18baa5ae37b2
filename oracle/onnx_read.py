"""TEST INFRASTRUCTURE ONLY: a restatement of the reference's ONNX reader.

What `load_onnx_memory` (crates/qppocr-core/src/onnx/parse.rs:550-749) takes
from a model's bytes, before its graph passes: the protobuf fields it reads,
how it widens tensors (float / double -> f32, every integer type -> i64), the
Constant folding into initializers (parse.rs:631-686) and the Identity
elimination (parse.rs:688-728).  The tests use it to check that the ONNX
files qppocr_b200.onnx_emit writes read back, field by field, as the graphs
and weights they were made from.  Nothing in the product imports it.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

DT_FLOAT, DT_UINT8, DT_INT8, DT_UINT16, DT_INT16, DT_INT32, DT_INT64 = 1, 2, 3, 4, 5, 6, 7
DT_BOOL, DT_DOUBLE = 9, 11


class ParseError(Exception):
    pass


class Reader:
    """parse.rs:26-137: a cursor over one length-delimited window."""

    def __init__(self, buf: bytes, start: int = 0, end: Optional[int] = None):
        self.buf = buf
        self.pos = start
        self.end = len(buf) if end is None else end

    def sub(self, s: int, l: int) -> "Reader":
        return Reader(self.buf, s, s + l)

    def eof(self) -> bool:
        return self.pos >= self.end

    def varint(self) -> int:
        v, shift = 0, 0
        while True:
            if self.pos >= self.end:
                raise ParseError("truncated varint")
            b = self.buf[self.pos]
            self.pos += 1
            v |= (b & 0x7F) << shift
            if not b & 0x80:
                return v & ((1 << 64) - 1)
            shift += 7
            if shift >= 64:
                raise ParseError("varint too long")

    def fixed32(self) -> int:
        if self.pos + 4 > self.end:
            raise ParseError("truncated fixed32")
        v = struct.unpack_from("<I", self.buf, self.pos)[0]
        self.pos += 4
        return v

    def fixed64(self) -> int:
        if self.pos + 8 > self.end:
            raise ParseError("truncated fixed64")
        v = struct.unpack_from("<Q", self.buf, self.pos)[0]
        self.pos += 8
        return v

    def bytes_(self) -> Tuple[int, int]:
        l = self.varint()
        s = self.pos
        if s + l > self.end:
            raise ParseError("truncated bytes")
        self.pos += l
        return s, l

    def str_at(self, s: int, l: int) -> str:
        return self.buf[s:s + l].decode("utf-8", errors="replace")

    def skip(self, wire: int) -> None:
        if wire == 0:
            self.varint()
        elif wire == 1:
            self.fixed64()
        elif wire == 2:
            self.bytes_()
        elif wire == 5:
            self.fixed32()
        else:
            raise ParseError(f"unsupported wire type {wire}")


def _i64(v: int) -> int:
    return v - (1 << 64) if v >= 1 << 63 else v


@dataclass
class Tensor:
    name: str = ""
    shape: List[int] = field(default_factory=list)
    dtype: str = "f32"  # "f32" or "i64", the two types the kernels take
    f32: Optional[np.ndarray] = None
    i64: List[int] = field(default_factory=list)


def parse_tensor(r: Reader) -> Tensor:
    """parse.rs:148-315."""
    t = Tensor()
    f32v: List[float] = []
    raw_dtype = DT_FLOAT
    while not r.eof():
        key = r.varint()
        fld, wire = key >> 3, key & 7
        if fld == 1:
            if wire == 2:
                s, l = r.bytes_()
                rd = r.sub(s, l)
                while not rd.eof():
                    t.shape.append(_i64(rd.varint()))
            else:
                t.shape.append(_i64(r.varint()))
        elif fld == 2:
            raw_dtype = r.varint()
        elif fld == 4:
            if wire == 2:
                s, l = r.bytes_()
                f32v.extend(np.frombuffer(r.buf, "<f4", l // 4, s).tolist())
            else:
                f32v.append(struct.unpack("<f", struct.pack("<I", r.fixed32()))[0])
        elif fld == 5:
            if wire == 2:
                s, l = r.bytes_()
                rd = r.sub(s, l)
                while not rd.eof():
                    t.i64.append(int(np.int32(np.uint32(rd.varint() & 0xFFFFFFFF))))
            elif wire == 0:
                t.i64.append(int(np.int32(np.uint32(r.varint() & 0xFFFFFFFF))))
            elif wire == 5:
                t.i64.append(int(np.int32(np.uint32(r.fixed32()))))
        elif fld == 7:
            if wire == 2:
                s, l = r.bytes_()
                rd = r.sub(s, l)
                while not rd.eof():
                    t.i64.append(_i64(rd.varint()))
            else:
                t.i64.append(_i64(r.varint()))
        elif fld == 8:
            s, l = r.bytes_()
            t.name = r.str_at(s, l)
        elif fld == 9:
            s, l = r.bytes_()
            raw = r.buf[s:s + l]
            if raw_dtype == DT_FLOAT:
                f32v.extend(np.frombuffer(raw, "<f4", l // 4).tolist())
            elif raw_dtype == DT_DOUBLE:
                f32v.extend(np.frombuffer(raw, "<f8", l // 8).astype(np.float32).tolist())
            elif raw_dtype == DT_INT64:
                t.i64.extend(np.frombuffer(raw, "<i8", l // 8).tolist())
            elif raw_dtype == DT_INT32:
                t.i64.extend(np.frombuffer(raw, "<i4", l // 4).tolist())
            elif raw_dtype in (DT_BOOL, DT_UINT8):
                t.i64.extend(np.frombuffer(raw, "u1", l).tolist())
            elif raw_dtype == DT_INT8:
                t.i64.extend(np.frombuffer(raw, "i1", l).tolist())
            elif raw_dtype == DT_UINT16:
                t.i64.extend(np.frombuffer(raw, "<u2", l // 2).tolist())
            elif raw_dtype == DT_INT16:
                t.i64.extend(np.frombuffer(raw, "<i2", l // 2).tolist())
            else:
                raise ParseError(f"raw_data: unsupported data_type {raw_dtype}")
        elif fld == 10:
            if wire == 2:
                s, l = r.bytes_()
                f32v.extend(np.frombuffer(r.buf, "<f8", l // 8, s).astype(np.float32).tolist())
            else:
                f32v.append(float(np.float32(struct.unpack("<d", struct.pack("<Q", r.fixed64()))[0])))
            if raw_dtype == DT_DOUBLE:
                raw_dtype = DT_FLOAT
        else:
            r.skip(wire)
    t.f32 = np.asarray(f32v, np.float32)
    t.dtype = "f32" if raw_dtype in (DT_FLOAT, DT_DOUBLE) else "i64"
    return t


@dataclass
class Attribute:
    name: str = ""
    f: Optional[float] = None
    i: Optional[int] = None
    s: Optional[str] = None
    tensor: Optional[Tensor] = None
    floats: List[float] = field(default_factory=list)
    ints: List[int] = field(default_factory=list)


def parse_attribute(r: Reader) -> Attribute:
    """parse.rs:317-374."""
    a = Attribute()
    while not r.eof():
        key = r.varint()
        fld, wire = key >> 3, key & 7
        if fld == 1:
            s, l = r.bytes_()
            a.name = r.str_at(s, l)
        elif fld == 2:
            a.f = struct.unpack("<f", struct.pack("<I", r.fixed32()))[0]
        elif fld == 3:
            a.i = _i64(r.varint())
        elif fld == 4:
            s, l = r.bytes_()
            a.s = r.str_at(s, l)
        elif fld == 5:
            s, l = r.bytes_()
            a.tensor = parse_tensor(r.sub(s, l))
        elif fld == 7:
            if wire == 2:
                s, l = r.bytes_()
                rd = r.sub(s, l)
                while not rd.eof():
                    a.floats.append(struct.unpack("<f", struct.pack("<I", rd.fixed32()))[0])
            else:
                a.floats.append(struct.unpack("<f", struct.pack("<I", r.fixed32()))[0])
        elif fld == 8:
            if wire == 2:
                s, l = r.bytes_()
                rd = r.sub(s, l)
                while not rd.eof():
                    a.ints.append(_i64(rd.varint()))
            else:
                a.ints.append(_i64(r.varint()))
        else:
            r.skip(wire)
    return a


@dataclass
class OnnxNode:
    op_type: str = ""
    name: str = ""
    inputs: List[str] = field(default_factory=list)
    outputs: List[str] = field(default_factory=list)
    attrs: List[Attribute] = field(default_factory=list)


def parse_node(r: Reader) -> OnnxNode:
    """parse.rs:376-408."""
    n = OnnxNode()
    while not r.eof():
        key = r.varint()
        fld, wire = key >> 3, key & 7
        if fld in (1, 2, 3, 4):
            s, l = r.bytes_()
            v = r.str_at(s, l)
            if fld == 1:
                n.inputs.append(v)
            elif fld == 2:
                n.outputs.append(v)
            elif fld == 3:
                n.name = v
            else:
                n.op_type = v
        elif fld == 5:
            s, l = r.bytes_()
            n.attrs.append(parse_attribute(r.sub(s, l)))
        else:
            r.skip(wire)
    return n


def _value_info(r: Reader, want_dims: bool):
    """parse.rs:410-501: the name, and for graph inputs the declared dims
    (dim_param or a missing value reads as 0, dynamic)."""
    name, dims = None, []
    while not r.eof():
        k = r.varint()
        f, w = k >> 3, k & 7
        if f == 1 and w == 2:
            s, l = r.bytes_()
            name = r.str_at(s, l)
            if not want_dims:
                return name, dims
        elif f == 2 and w == 2 and want_dims:
            s, l = r.bytes_()
            ty = r.sub(s, l)
            while not ty.eof():
                k2 = ty.varint()
                if (k2 >> 3, k2 & 7) == (1, 2):
                    s2, l2 = ty.bytes_()
                    tt = ty.sub(s2, l2)
                    while not tt.eof():
                        k3 = tt.varint()
                        if (k3 >> 3, k3 & 7) == (2, 2):
                            s3, l3 = tt.bytes_()
                            shp = tt.sub(s3, l3)
                            while not shp.eof():
                                k4 = shp.varint()
                                if (k4 >> 3, k4 & 7) == (1, 2):
                                    s4, l4 = shp.bytes_()
                                    dim = shp.sub(s4, l4)
                                    v = 0
                                    while not dim.eof():
                                        k5 = dim.varint()
                                        if (k5 >> 3, k5 & 7) == (1, 0):
                                            v = _i64(dim.varint())
                                        elif (k5 >> 3, k5 & 7) == (2, 2):
                                            dim.bytes_()
                                            v = 0
                                        else:
                                            dim.skip(k5 & 7)
                                    dims.append(v)
                                else:
                                    shp.skip(k4 & 7)
                        else:
                            tt.skip(k3 & 7)
                else:
                    ty.skip(k2 & 7)
        else:
            r.skip(w)
    return name, dims


@dataclass
class OnnxModel:
    ir_version: int = 0
    producer_name: str = ""
    producer_version: str = ""
    opset_version: int = 0
    graph_name: str = ""
    nodes: List[OnnxNode] = field(default_factory=list)
    inputs: List[str] = field(default_factory=list)
    input_dims: List[List[int]] = field(default_factory=list)
    outputs: List[str] = field(default_factory=list)
    initializers: Dict[str, Tensor] = field(default_factory=dict)
    metadata: Dict[str, str] = field(default_factory=dict)


def _parse_graph(r: Reader, g: OnnxModel) -> None:
    """parse.rs:503-548: nodes and initializers are collected first and
    parsed after the scan, in file order."""
    node_chunks, init_chunks = [], []
    while not r.eof():
        key = r.varint()
        fld, wire = key >> 3, key & 7
        if wire != 2:
            r.skip(wire)
            continue
        s, l = r.bytes_()
        if fld == 1:
            node_chunks.append((s, l))
        elif fld == 2:
            g.graph_name = r.str_at(s, l)
        elif fld == 5:
            init_chunks.append((s, l))
        elif fld == 11:
            nm, dims = _value_info(r.sub(s, l), True)
            if nm is not None:
                g.inputs.append(nm)
                g.input_dims.append(dims)
        elif fld == 12:
            nm, _ = _value_info(r.sub(s, l), False)
            if nm is not None:
                g.outputs.append(nm)
    for s, l in node_chunks:
        g.nodes.append(parse_node(r.sub(s, l)))
    for s, l in init_chunks:
        t = parse_tensor(r.sub(s, l))
        g.initializers[t.name] = t


def load_onnx_memory(data: bytes) -> OnnxModel:
    """parse.rs:550-729, up to (not including) the structural graph passes
    that follow (parse.rs:731-747; qppocr_b200.graph.optimize restates them)."""
    r = Reader(data)
    g = OnnxModel()
    while not r.eof():
        key = r.varint()
        fld, wire = key >> 3, key & 7
        if wire != 2:
            if wire == 0:
                v = r.varint()
                if fld == 1:
                    g.ir_version = _i64(v)
            else:
                r.skip(wire)
            continue
        s, l = r.bytes_()
        if fld == 2:
            g.producer_name = r.str_at(s, l)
        elif fld == 3:
            g.producer_version = r.str_at(s, l)
        elif fld == 8:
            orr = r.sub(s, l)
            ver, dom = 0, "ai.onnx"
            while not orr.eof():
                k = orr.varint()
                if (k >> 3, k & 7) == (1, 2):
                    s2, l2 = orr.bytes_()
                    dom = orr.str_at(s2, l2)
                elif (k >> 3, k & 7) == (2, 0):
                    ver = _i64(orr.varint())
                else:
                    orr.skip(k & 7)
            if dom in ("ai.onnx", "") or g.opset_version == 0:
                g.opset_version = ver
        elif fld == 7:
            _parse_graph(r.sub(s, l), g)
        elif fld == 14:
            er = r.sub(s, l)
            k_, v_ = "", ""
            while not er.eof():
                k2 = er.varint()
                if (k2 >> 3, k2 & 7) == (1, 2):
                    s2, l2 = er.bytes_()
                    k_ = er.str_at(s2, l2)
                elif (k2 >> 3, k2 & 7) == (2, 2):
                    s2, l2 = er.bytes_()
                    v_ = er.str_at(s2, l2)
                else:
                    er.skip(k2 & 7)
            if k_:
                g.metadata[k_] = v_
    if not g.nodes:
        raise ParseError("model has no nodes (parse failure?)")
    # Constant -> initializer (parse.rs:631-686)
    kept = []
    for n in g.nodes:
        if n.op_type == "Constant":
            out = n.outputs[0]
            t = None
            for a in n.attrs:
                if a.name == "value" and a.tensor is not None:
                    t = a.tensor
                    t.name = out
                elif a.name == "value_float":
                    t = Tensor(out, [], "f32", np.asarray([a.f or 0.0], np.float32))
                elif a.name == "value_floats":
                    t = Tensor(out, [], "f32", np.asarray(a.floats, np.float32))
                elif a.name in ("value_int", "value_ints"):
                    t = Tensor(out, [], "i64", np.zeros(0, np.float32), list(a.ints))
                if t is not None:
                    break
            if t is not None:
                g.initializers[out] = t
                continue
        kept.append(n)
    g.nodes = kept
    # Identity elimination (parse.rs:688-728)
    alias = {n.outputs[0]: n.inputs[0] for n in g.nodes if n.op_type == "Identity" and n.inputs and n.outputs}
    if alias:
        def resolve(nm):
            for _ in range(64):
                if nm not in alias:
                    break
                nm = alias[nm]
            return nm
        out = []
        for n in g.nodes:
            if n.op_type == "Identity":
                continue
            n.inputs = [resolve(i) if i else i for i in n.inputs]
            out.append(n)
        g.outputs = [resolve(o) for o in g.outputs]
        g.nodes = out
    return g
