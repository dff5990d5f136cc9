#!/usr/bin/env python3
"""Generate the ONNX fixtures under tests/golden/ with the REFERENCE's own exporter.

Run in a container that holds the reference checkout (not needed on the GPU box):

    python tests/golden/make_onnx.py --reference /path/to/katago-rs

Per net in NETS: the seeded `.bin` net (katago_cuda.netgen) is parsed by the reference's parser and turned into a
graph by its `build_onnx` (tools/bin2onnx/bin2onnx.py:1571-1615), exactly as `bin2onnx.py` does for the files its
burn backend is generated from. The Python package `onnx` is absent here, so the recording stand-in of
make_golden.py takes the nodes, initializers and metadata that build_onnx emits, and this script writes them as an
ONNX ModelProto in the protobuf wire format (field numbers of the public onnx.proto schema). Nothing of the graph
construction is re-implemented. The outputs are `<net>.onnx`; tests/test_onnx_load.py loads them through the C ABI
and compares them with the `.bin` nets they were made from.
"""

from __future__ import annotations

import argparse
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "katago-rs_b200", "python"))

from katago_cuda import netgen  # noqa: E402
from make_golden import install_onnx_stub  # noqa: E402

# every block kind, RoPE flavour (learnable, fixed, none), grouped-query attention, trunk tip (BN, RMSNorm per
# point, spatial RMSNorm), policy channels 1 / 2 / 4, the v15+ pass MLP and the metadata encoder
NETS = ["tiny-resnet", "tiny-nbt", "tiny-v15-meta", "tiny-tf-learn", "tiny-tf-spatial"]


# ---- protobuf wire format ----

def _varint(v: int) -> bytes:
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


def _key(field: int, wire: int) -> bytes:
    return _varint((field << 3) | wire)


def _len(field: int, payload: bytes) -> bytes:
    return _key(field, 2) + _varint(len(payload)) + payload


def _str(field: int, s: str) -> bytes:
    return _len(field, s.encode())


def _int(field: int, v: int) -> bytes:
    return _key(field, 0) + _varint(int(v))


def _packed_ints(field: int, vals) -> bytes:
    return _len(field, b"".join(_varint(int(v)) for v in vals))


def tensor_proto(name: str, arr: np.ndarray) -> bytes:
    """TensorProto: dims (1), data_type (2: 1 FLOAT, 7 INT64), name (8), raw_data (9)."""
    arr = np.ascontiguousarray(arr)
    if arr.dtype.kind == "f":
        dtype, raw = 1, arr.astype("<f4").tobytes()
    elif arr.dtype.kind in "iu":
        dtype, raw = 7, arr.astype("<i8").tobytes()
    else:
        raise TypeError(f"{name}: {arr.dtype}")
    out = b"".join(_int(1, d) for d in arr.shape)
    return out + _int(2, dtype) + _str(8, name) + _len(9, raw)


def attribute_proto(name: str, value) -> bytes:
    """AttributeProto: name (1), f (2), i (3), ints (8), type (20: 1 FLOAT, 2 INT, 7 INTS)."""
    out = _str(1, name)
    if isinstance(value, (list, tuple)):
        return out + b"".join(_int(8, v) for v in value) + _int(20, 7)
    if isinstance(value, float):
        return out + _key(2, 5) + struct.pack("<f", value) + _int(20, 1)
    return out + _int(3, int(value)) + _int(20, 2)


def node_proto(nd) -> bytes:
    """NodeProto: input (1), output (2), name (3), op_type (4), attribute (5)."""
    out = b"".join(_str(1, i) for i in nd.input) + b"".join(_str(2, o) for o in nd.output)
    out += _str(3, nd.name or nd.output[0]) + _str(4, nd.op_type)
    return out + b"".join(_len(5, attribute_proto(k, v)) for k, v in nd.attrs.items())


def model_proto(model) -> bytes:
    """ModelProto: ir_version (1), producer_name (2), graph (7), opset_import (8), metadata_props (14)."""
    g = model.graph
    graph = b"".join(_len(1, node_proto(nd)) for nd in g.node)
    graph += _str(2, g.name)
    graph += b"".join(_len(5, tensor_proto(i.name, i.array)) for i in g.initializer)
    for (args, _kw) in g.input:  # ValueInfoProto: name (1)
        graph += _len(11, _str(1, args[0]))
    for (args, _kw) in g.output:
        graph += _len(12, _str(1, args[0]))
    out = _int(1, 8) + _str(2, "katago-rs bin2onnx") + _len(7, graph) + _len(8, _str(1, "") + _int(2, 17))
    for e in model.metadata_props:  # StringStringEntryProto: key (1), value (2)
        out += _len(14, _str(1, e.key) + _str(2, e.value))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="katago-rs checkout (reads tools/bin2onnx/bin2onnx.py)")
    ap.add_argument("--only", nargs="*", help="subset of nets")
    args = ap.parse_args()
    install_onnx_stub()
    sys.path.insert(0, os.path.join(args.reference, "tools", "bin2onnx"))
    import bin2onnx as b2o  # the reference's parser and graph builder

    for name in NETS:
        if args.only and name not in args.only:
            continue
        desc = b2o.parse_model(b2o.ModelReader(netgen.net_bytes(name), True))
        data = model_proto(b2o.build_onnx(desc, pos_len=19))
        with open(os.path.join(HERE, f"{name}.onnx"), "wb") as f:
            f.write(data)
        print(f"{name}.onnx: {len(data)} bytes", flush=True)


if __name__ == "__main__":
    main()
