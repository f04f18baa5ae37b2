"""The ONNX files of the synthetic nets (qppocr_b200.onnx_emit) read back as
the graphs and weights they were made from:

* through the oracle's restatement of the reference's reader
  (crates/qppocr-core/src/onnx/parse.rs:550-729): every node, attribute,
  graph input (with its declared dims), output, and weight bit for bit;
* through the protobuf runtime with the ONNX message schema (field numbers of
  onnx.proto), an independent decoder of the same bytes;
* and the read-back graph, after the loader's graph passes, computes the same
  outputs on the oracle as the original graph, bit for bit.
"""
import struct
import zlib

import numpy as np
import pytest

import oracle as orc
import qppocr_b200 as q
from oracle.onnx_read import load_onnx_memory
from qppocr_b200 import nets, onnx_emit
from qppocr_b200.graph import Graph, Node

NETS = {"det": nets.build_det, "rec": nets.build_rec, "cls": nets.build_cls, "block": nets.build_block}


def _attr_value(a, like):
    if isinstance(like, str):
        return a.s
    if isinstance(like, float):
        return a.f
    if isinstance(like, (list, tuple)):
        return a.ints
    return a.i


@pytest.mark.parametrize("net", sorted(NETS))
def test_reference_reader_reads_back_graph_and_weights(net):
    g, w = NETS[net]()
    m = load_onnx_memory(onnx_emit.model_bytes(g, w, net))
    assert m.ir_version == onnx_emit.IR_VERSION and m.opset_version == onnx_emit.OPSET
    assert m.graph_name == net and m.producer_name == "qppocr_b200.nets"
    assert m.inputs == g.inputs and m.outputs == g.outputs
    assert m.input_dims == [list(d) for d in g.input_dims]
    assert len(m.nodes) == len(g.nodes)
    for a, b in zip(m.nodes, g.nodes):
        assert (a.op_type, a.name, a.inputs, a.outputs) == (b.op_type, b.name, b.inputs, b.outputs)
        got = {x.name: x for x in a.attrs}
        assert set(got) == set(b.attrs), b.name
        for k, v in b.attrs.items():
            rv = _attr_value(got[k], v)
            if isinstance(v, float):
                assert np.float32(rv) == np.float32(v), (b.name, k)
            elif isinstance(v, (list, tuple)):
                assert list(rv) == list(v), (b.name, k)
            else:
                assert rv == v, (b.name, k)
    used = {i for n in g.nodes for i in n.inputs if i}
    assert set(m.initializers) == {k for k in w if k in used}
    for k, t in m.initializers.items():
        ref = np.asarray(w[k])
        assert t.shape == list(ref.shape), k
        if ref.dtype.kind == "f":
            assert t.dtype == "f32"
            assert np.array_equal(t.f32.view(np.uint32), ref.astype(np.float32).ravel().view(np.uint32)), k
        else:
            assert t.dtype == "i64" and t.i64 == ref.astype(np.int64).ravel().tolist(), k


def test_rec_dictionary_metadata_matches_head():
    g, w = nets.build_rec()
    classes = w[[n for n in g.nodes if n.op_type == "MatMul"][-1].inputs[1]].shape[1]
    text = onnx_emit.synthetic_dictionary(classes - 2)
    m = load_onnx_memory(onnx_emit.model_bytes(g, w, "rec", {"character": text}))
    # engine.rs:447-470: blank, one entry per line, then a space
    charset = ["blank"] + m.metadata["character"].split("\n") + [" "]
    assert len(charset) == classes
    assert len(set(charset[1:-1])) == classes - 2 and all(len(c) == 1 for c in charset[1:-1])


def _onnx_classes():
    """The ONNX messages the emitter writes, declared with onnx.proto's field
    numbers, as protobuf runtime classes."""
    from google.protobuf import descriptor_pb2, descriptor_pool, message_factory

    F = descriptor_pb2.FieldDescriptorProto
    fd = descriptor_pb2.FileDescriptorProto(name="onnx_subset.proto", package="onnx_subset", syntax="proto2")

    def msg(name, fields):
        m = fd.message_type.add(name=name)
        for (fname, num, typ, label, tname) in fields:
            f = m.field.add(name=fname, number=num, type=typ, label=label)
            if tname:
                f.type_name = ".onnx_subset." + tname
        return m

    O, R = F.LABEL_OPTIONAL, F.LABEL_REPEATED
    msg("TensorProto", [("dims", 1, F.TYPE_INT64, R, None), ("data_type", 2, F.TYPE_INT32, O, None),
                        ("name", 8, F.TYPE_STRING, O, None), ("raw_data", 9, F.TYPE_BYTES, O, None)])
    msg("AttributeProto", [("name", 1, F.TYPE_STRING, O, None), ("f", 2, F.TYPE_FLOAT, O, None),
                           ("i", 3, F.TYPE_INT64, O, None), ("s", 4, F.TYPE_BYTES, O, None),
                           ("floats", 7, F.TYPE_FLOAT, R, None), ("ints", 8, F.TYPE_INT64, R, None),
                           ("type", 20, F.TYPE_INT32, O, None)])
    msg("NodeProto", [("input", 1, F.TYPE_STRING, R, None), ("output", 2, F.TYPE_STRING, R, None),
                      ("name", 3, F.TYPE_STRING, O, None), ("op_type", 4, F.TYPE_STRING, O, None),
                      ("attribute", 5, F.TYPE_MESSAGE, R, "AttributeProto")])
    msg("Dimension", [("dim_value", 1, F.TYPE_INT64, O, None), ("dim_param", 2, F.TYPE_STRING, O, None)])
    msg("TensorShapeProto", [("dim", 1, F.TYPE_MESSAGE, R, "Dimension")])
    msg("TensorTypeProto", [("elem_type", 1, F.TYPE_INT32, O, None),
                            ("shape", 2, F.TYPE_MESSAGE, O, "TensorShapeProto")])
    msg("TypeProto", [("tensor_type", 1, F.TYPE_MESSAGE, O, "TensorTypeProto")])
    msg("ValueInfoProto", [("name", 1, F.TYPE_STRING, O, None), ("type", 2, F.TYPE_MESSAGE, O, "TypeProto")])
    msg("GraphProto", [("node", 1, F.TYPE_MESSAGE, R, "NodeProto"), ("name", 2, F.TYPE_STRING, O, None),
                       ("initializer", 5, F.TYPE_MESSAGE, R, "TensorProto"),
                       ("input", 11, F.TYPE_MESSAGE, R, "ValueInfoProto"),
                       ("output", 12, F.TYPE_MESSAGE, R, "ValueInfoProto")])
    msg("OperatorSetIdProto", [("domain", 1, F.TYPE_STRING, O, None), ("version", 2, F.TYPE_INT64, O, None)])
    msg("StringStringEntryProto", [("key", 1, F.TYPE_STRING, O, None), ("value", 2, F.TYPE_STRING, O, None)])
    msg("ModelProto", [("ir_version", 1, F.TYPE_INT64, O, None), ("producer_name", 2, F.TYPE_STRING, O, None),
                       ("producer_version", 3, F.TYPE_STRING, O, None),
                       ("graph", 7, F.TYPE_MESSAGE, O, "GraphProto"),
                       ("opset_import", 8, F.TYPE_MESSAGE, R, "OperatorSetIdProto"),
                       ("metadata_props", 14, F.TYPE_MESSAGE, R, "StringStringEntryProto")])
    pool = descriptor_pool.DescriptorPool()
    pool.Add(fd)
    return message_factory.GetMessageClass(pool.FindMessageTypeByName("onnx_subset.ModelProto"))


@pytest.mark.parametrize("net", ["cls", "block"])
def test_protobuf_runtime_decodes_the_same_model(net):
    g, w = NETS[net]()
    data = onnx_emit.model_bytes(g, w, net, {"k": "v"})
    m = _onnx_classes()()
    m.ParseFromString(data)
    assert m.SerializeToString() == data  # canonical encoding: nothing unknown, nothing reordered
    assert m.ir_version == onnx_emit.IR_VERSION and m.opset_import[0].version == onnx_emit.OPSET
    assert m.metadata_props[0].key == "k" and m.metadata_props[0].value == "v"
    assert [n.op_type for n in m.graph.node] == [n.op_type for n in g.nodes]
    for pn, n in zip(m.graph.node, g.nodes):
        assert list(pn.input) == n.inputs and list(pn.output) == n.outputs
        for pa in pn.attribute:
            v = n.attrs[pa.name]
            if pa.type == onnx_emit.AT_INTS:
                assert list(pa.ints) == list(v)
            elif pa.type == onnx_emit.AT_INT:
                assert pa.i == v
            elif pa.type == onnx_emit.AT_FLOAT:
                assert np.float32(pa.f) == np.float32(v)
            else:
                assert pa.type == onnx_emit.AT_STRING and pa.s.decode() == v
    for t in m.graph.initializer:
        ref = np.asarray(w[t.name])
        assert list(t.dims) == list(ref.shape)
        dt = "<f4" if t.data_type == onnx_emit.DT_FLOAT else "<i8"
        assert np.array_equal(np.frombuffer(t.raw_data, dt), ref.ravel().astype(dt))
    dims = [d.dim_value if d.HasField("dim_value") else 0 for d in m.graph.input[0].type.tensor_type.shape.dim]
    assert dims == list(g.input_dims[0])


def _graph_from_onnx(m):
    nodes = []
    for n in m.nodes:
        attrs = {}
        for a in n.attrs:
            if a.s is not None:
                attrs[a.name] = a.s
            elif a.f is not None:
                attrs[a.name] = float(a.f)
            elif a.ints:
                attrs[a.name] = list(a.ints)
            else:
                attrs[a.name] = a.i
        nodes.append(Node(n.op_type, n.name, list(n.inputs), list(n.outputs), attrs))
    w = {}
    for k, t in m.initializers.items():
        w[k] = (t.f32.reshape(t.shape) if t.dtype == "f32" else np.asarray(t.i64, np.int64).reshape(t.shape))
    return Graph(nodes, list(m.inputs), list(m.outputs), [list(d) for d in m.input_dims]), w


@pytest.mark.parametrize("net,x", [("cls", lambda: nets.cls_input(2)),
                                   ("block", lambda: nets.block_input(0, (1, 64, 24, 40))),
                                   ("det", lambda: nets.det_input(1, 64, 96))])
def test_read_back_graph_computes_the_same_outputs(net, x):
    g, w = NETS[net]()
    g2, w2 = _graph_from_onnx(load_onnx_memory(onnx_emit.model_bytes(g, w, net)))
    xin = x()
    ref = orc.run_graph(q.optimize(g, w), w, {"x": xin})[0]
    got = orc.run_graph(q.optimize(g2, w2), w2, {"x": xin})[0]
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def _png_pixels(data: bytes) -> np.ndarray:
    assert data[:8] == b"\x89PNG\r\n\x1a\n"
    pos, idat, hdr = 8, b"", None
    while pos < len(data):
        (n,) = struct.unpack(">I", data[pos:pos + 4])
        tag, body = data[pos + 4:pos + 8], data[pos + 8:pos + 8 + n]
        (crc,) = struct.unpack(">I", data[pos + 8 + n:pos + 12 + n])
        assert crc == zlib.crc32(tag + body) & 0xFFFFFFFF
        if tag == b"IHDR":
            hdr = struct.unpack(">IIBBBBB", body)
        elif tag == b"IDAT":
            idat += body
        pos += 12 + n
    w, h, depth, ctype = hdr[:4]
    assert depth == 8 and ctype == 2
    rows = np.frombuffer(zlib.decompress(idat), np.uint8).reshape(h, 1 + 3 * w)
    assert not rows[:, 0].any()  # filter type 0 on every row
    return rows[:, 1:].reshape(h, w, 3)


def test_model_dir_layout_and_images(tmp_path):
    paths = onnx_emit.write_model_dir(str(tmp_path), "small", n_images=2, hw=40)
    rel = sorted(p[len(str(tmp_path)) + 1:] for p in paths)
    assert rel == ["cls.onnx", "images/img_0000.png", "images/img_0001.png", "small/det.onnx", "small/rec.onnx"]
    imgs = list(onnx_emit.synthetic_images(2, 40, 40))
    for k in range(2):
        got = _png_pixels((tmp_path / "images" / f"img_{k:04d}.png").read_bytes())
        assert np.array_equal(got, imgs[k])
    m = load_onnx_memory((tmp_path / "small" / "rec.onnx").read_bytes())
    assert "character" in m.metadata
