#!/usr/bin/env python3
"""Generate the golden fixtures under tests/golden/ from the REFERENCE's own graph.

Run in a container that holds the reference checkout (not needed on the GPU box):

    python tests/golden/make_golden.py --reference /path/to/katago-rs

What it does, per net in NETS below:
 1. writes the seeded random-init net with this repo's `.bin` writer (katago_cuda.netgen);
 2. parses those bytes with the reference's parser (`tools/bin2onnx/bin2onnx.py` `parse_model`), which pins the
    writer to the file format the reference reads;
 3. builds the reference's forward graph with its `build_onnx` / `GraphBuilder` (bin2onnx.py:1088-1615). The
    Python package `onnx` is absent here, so a minimal stand-in records the nodes and initializers that
    GraphBuilder emits; nothing of the graph construction is re-implemented;
 4. executes that node list with a small numpy interpreter of the ONNX operators it uses (standard ONNX opset-17
    semantics), in float64, on seeded synthetic inputs;
 5. saves inputs, outputs and the reference ModelDesc summary to `<net>.npz` / `descs.json`.

The graph is what burn-onnx turns into the reference's `flex` forward pass, so these outputs are the reference
semantics evaluated in float64. The C++ oracle (oracle/) is checked against them by tests/test_oracle_golden.py.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "katago-rs_b200", "python"))

from katago_cuda import inputs as kinputs  # noqa: E402
from katago_cuda import netgen  # noqa: E402

# name -> (batch, board sizes, input seed, rich inputs)
NETS = {
    "tiny-resnet": (3, (19, 9, 13), 11, True),
    "tiny-nbt": (3, (19, 13, 9), 12, True),
    "tiny-v15-meta": (3, (9, 19, 13), 13, True),
    "tiny-tf-learn": (3, (19, 9, 13), 14, True),
    "tiny-tf-spatial": (3, (13, 19, 9), 15, True),
    "small-nbt": (2, (19, 9), 16, False),
    "small-tf": (2, (19, 13), 17, False),
    "b10c128": (2, (19,), 18, False),
    "b18c384nbt": (1, (19,), 19, False),
    "b10c384h6": (1, (19,), 20, False),
    "tf3-b11c768": (2, (19, 13), 21, False),
    "gqa-tf": (3, (19, 9, 13), 22, True),
    "wide-nbt": (3, (13, 19, 9), 23, True),
}


# ---------------------------------------------------------------------------------------------------------------
# Minimal stand-in for the `onnx` package: records what GraphBuilder emits.
# ---------------------------------------------------------------------------------------------------------------

class _Node:
    def __init__(self, op, inputs, outputs, name=None, **attrs):
        self.op_type = op
        self.input = list(inputs)
        self.output = list(outputs)
        self.name = name
        self.attrs = attrs


class _Init:
    def __init__(self, arr, name):
        self.name = name
        self.array = np.array(arr)


class _Props(list):
    def add(self):
        e = types.SimpleNamespace(key=None, value=None)
        self.append(e)
        return e


class _Model:
    def __init__(self, graph):
        self.graph = graph
        self.metadata_props = _Props()
        self.ir_version = None


def install_onnx_stub():
    onnx = types.ModuleType("onnx")
    helper = types.ModuleType("onnx.helper")
    numpy_helper = types.ModuleType("onnx.numpy_helper")
    helper.make_node = lambda op, inputs, outputs, name=None, **attrs: _Node(op, inputs, outputs, name, **attrs)
    helper.make_tensor_value_info = lambda *a, **k: (a, k)
    helper.make_graph = lambda nodes, name, inputs, outputs, inits: types.SimpleNamespace(
        node=nodes, name=name, input=inputs, output=outputs, initializer=inits)
    helper.make_model = lambda graph, **k: _Model(graph)
    helper.make_opsetid = lambda *a: a
    numpy_helper.from_array = lambda arr, name: _Init(arr, name)
    onnx.helper = helper
    onnx.numpy_helper = numpy_helper
    onnx.TensorProto = types.SimpleNamespace(FLOAT=1)
    onnx.ModelProto = _Model
    sys.modules["onnx"] = onnx
    sys.modules["onnx.helper"] = helper
    sys.modules["onnx.numpy_helper"] = numpy_helper


# ---------------------------------------------------------------------------------------------------------------
# numpy interpreter of the ONNX operators GraphBuilder uses (ONNX opset 17 semantics)
# ---------------------------------------------------------------------------------------------------------------

def _conv(x, w, pads, dilations):
    n, c, h, wd = x.shape
    m, c2, kh, kw = w.shape
    assert c == c2
    pt, pl, pb, pr = pads
    dy, dx = dilations
    xp = np.zeros((n, c, h + pt + pb, wd + pl + pr), x.dtype)
    xp[:, :, pt:pt + h, pl:pl + wd] = x
    oh = h + pt + pb - dy * (kh - 1)
    ow = wd + pl + pr - dx * (kw - 1)
    out = np.zeros((n, m, oh, ow), x.dtype)
    for ky in range(kh):
        for kx in range(kw):
            patch = xp[:, :, ky * dy:ky * dy + oh, kx * dx:kx * dx + ow]      # [n,c,oh,ow]
            out += np.einsum("nchw,mc->nmhw", patch, w[:, :, ky, kx], optimize=True)
    return out


def run_graph(graph, feeds, dtype):
    env = {k: np.asarray(v, dtype) for k, v in feeds.items()}
    for ini in graph.initializer:
        a = ini.array
        env[ini.name] = a.astype(dtype) if a.dtype.kind == "f" else a
    for nd in graph.node:
        ins = [env[i] for i in nd.input]
        a = nd.attrs
        op = nd.op_type
        if op == "Conv":
            y = _conv(ins[0], ins[1], a["pads"], a["dilations"])
        elif op == "Relu":
            y = np.maximum(ins[0], 0)
        elif op == "Softplus":
            y = np.logaddexp(0, ins[0])
        elif op == "Tanh":
            y = np.tanh(ins[0])
        elif op == "Exp":
            with np.errstate(over="ignore"):
                y = np.exp(ins[0])
        elif op == "Sqrt":
            y = np.sqrt(ins[0])
        elif op == "Mul":
            y = ins[0] * ins[1]
        elif op == "Add":
            y = ins[0] + ins[1]
        elif op == "Sub":
            y = ins[0] - ins[1]
        elif op == "Div":
            y = ins[0] / ins[1]
        elif op == "MatMul":
            y = np.matmul(ins[0], ins[1])
        elif op == "Reshape":
            shape = [int(s) for s in ins[1]]
            y = ins[0].reshape(shape)
        elif op == "Slice":
            starts, ends, axes = (list(map(int, v)) for v in ins[1:4])
            sl = [slice(None)] * ins[0].ndim
            for s, e, ax in zip(starts, ends, axes):
                sl[ax] = slice(s, e)
            y = ins[0][tuple(sl)]
        elif op == "ReduceSum":
            axes = tuple(int(v) for v in ins[1])
            y = np.sum(ins[0], axis=axes, keepdims=bool(a.get("keepdims", 1)))
        elif op == "ReduceMax":
            y = np.max(ins[0], axis=tuple(a["axes"]), keepdims=bool(a.get("keepdims", 1)))
        elif op == "Concat":
            y = np.concatenate(ins, axis=a["axis"])
        elif op == "Transpose":
            y = np.transpose(ins[0], a["perm"])
        elif op == "Softmax":
            ax = a.get("axis", -1)
            z = ins[0] - np.max(ins[0], axis=ax, keepdims=True)
            e = np.exp(z)
            y = e / np.sum(e, axis=ax, keepdims=True)
        else:
            raise NotImplementedError(op)
        if y.dtype.kind == "f":
            y = y.astype(dtype, copy=False)
        env[nd.output[0]] = y
    return {k: env[k] for k in ("policy", "value", "scorevalue", "ownership")}


def desc_summary(b2o, desc):
    t = desc.trunk
    return {
        "name": desc.name,
        "modelVersion": desc.model_version,
        "numInputChannels": desc.num_input_channels,
        "numInputGlobalChannels": desc.num_input_global_channels,
        "numInputMetaChannels": desc.num_input_meta_channels,
        "metaEncoderVersion": desc.meta_encoder_version,
        "numPolicyChannels": desc.num_policy_channels,
        "numValueChannels": desc.num_value_channels,
        "numScoreValueChannels": desc.num_score_value_channels,
        "numOwnershipChannels": desc.num_ownership_channels,
        "trunkNumBlocks": t.num_blocks,
        "trunkNumChannels": t.trunk_num_channels,
        "trunkNormKind": t.trunk_norm_kind,
        "numParameters": int(b2o.num_parameters(desc)),
        "trunkSpatialConvDepth": float(b2o.spatial_conv_depth(t)),
        "hasAnyTransformerBlocks": int(desc.has_any_transformer_blocks),
        "hasAnyNestedBottleneckBlocks": int(b2o.has_any_nested_bottleneck_blocks(desc)),
        "postProcess": [desc.post_process_params.td_score_multiplier, desc.post_process_params.score_mean_multiplier,
                        desc.post_process_params.score_stdev_multiplier, desc.post_process_params.lead_multiplier,
                        desc.post_process_params.variance_time_multiplier,
                        desc.post_process_params.shortterm_value_error_multiplier,
                        desc.post_process_params.shortterm_score_error_multiplier],
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="katago-rs checkout (reads tools/bin2onnx/bin2onnx.py)")
    ap.add_argument("--only", nargs="*", help="subset of nets")
    args = ap.parse_args()

    install_onnx_stub()
    sys.path.insert(0, os.path.join(args.reference, "tools", "bin2onnx"))
    import bin2onnx as b2o  # the reference's parser and graph builder

    descs = {}
    path = os.path.join(HERE, "descs.json")
    if os.path.exists(path):
        with open(path) as f:
            descs = json.load(f)
    for name, (n, sizes, seed, rich) in NETS.items():
        if args.only and name not in args.only:
            continue
        data = netgen.net_bytes(name)
        desc = b2o.parse_model(b2o.ModelReader(data, True))
        model = b2o.build_onnx(desc, pos_len=19)
        nm = desc.num_input_meta_channels
        spatial, glob, meta, bsz = kinputs.synthetic_inputs(n, seed, sizes, desc.num_input_channels,
                                                            desc.num_input_global_channels, nm, rich)
        feeds = {"bin_input": spatial, "global_input": glob}
        if nm:
            feeds["meta_input"] = meta
        out = run_graph(model.graph, feeds, np.float64)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), bin_input=spatial, global_input=glob,
                            meta_input=meta, board_sizes=bsz, **{k: v for k, v in out.items()})
        s = desc_summary(b2o, desc)
        s["sha256"] = hashlib.sha256(data).hexdigest()
        s["batch"] = n
        s["nodes"] = len(model.graph.node)
        descs[name] = s
        print(f"{name}: {len(model.graph.node)} nodes, policy |max| {np.abs(out['policy']).max():.3f}, "
              f"value {out['value'][0]}, sha {s['sha256'][:12]}", flush=True)
    with open(path, "w") as f:
        json.dump(descs, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
