"""GPU parity: the CUDA forward pass (through the C ABI) against the golden fixtures (the reference graph in float64)
and the CPU oracle, at the tolerances north_star states: max-abs 1e-4 in f32 mode, 2e-2 in f16/bf16 mode on policy
logits, value/score and ownership."""

import json
import os

import numpy as np
import pytest

import katago_cuda as kc
from katago_cuda import inputs, netgen
from oracle.oracle import OracleNet

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
NAMES = sorted(json.load(open(os.path.join(GOLDEN, "descs.json"))))
TOL = {kc.PRECISION_F32: 1e-4, kc.PRECISION_F16: 2e-2, kc.PRECISION_BF16: 2e-2}
KEYS = ("policy", "value", "scorevalue", "ownership")

_HANDLES = {}


def handle(name, precision, max_batch):
    key = (name, precision, max_batch)
    if key not in _HANDLES:
        m = kc.Model(netgen.net_bytes(name))
        ctx = kc.Context(m, gpu_idxs=[0], precision=precision)
        _HANDLES[key] = kc.Handle(ctx, max_batch=max_batch, gpu_idx=0)
    return _HANDLES[key]


def half_precision(name):
    d = json.load(open(os.path.join(GOLDEN, "descs.json")))[name]
    return kc.PRECISION_BF16 if d["hasAnyTransformerBlocks"] else kc.PRECISION_F16


def max_err(got, want):
    return {k: float(np.abs(got[k] - want[k]).max()) for k in KEYS}


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("mode", ["f32", "half"])
def test_golden(name, mode):
    g = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    prec = kc.PRECISION_F32 if mode == "f32" else half_precision(name)
    h = handle(name, prec, 8)
    got = h.forward(g["bin_input"], g["global_input"], g["meta_input"])
    errs = max_err(got, {k: g[k] for k in KEYS})
    for k in KEYS:
        assert np.all(np.isfinite(got[k])), k
        assert errs[k] <= TOL[prec], (name, mode, errs)


@pytest.mark.parametrize("name,prec", [("small-nbt", kc.PRECISION_F16), ("tiny-nbt", kc.PRECISION_F32),
                                       ("small-tf", kc.PRECISION_BF16), ("tiny-tf-learn", kc.PRECISION_F32),
                                       ("tiny-v15-meta", kc.PRECISION_F16), ("gqa-tf", kc.PRECISION_F32)])
def test_oracle_mixed_boards(name, prec):
    """Batches of mixed 9x9 / 13x13 / 19x19 boards (masked BN, masked pooling and the max-pool paths), larger than one
    128-row tile, against the float32 oracle."""
    n = 37
    m = kc.Model(netgen.net_bytes(name))
    spatial, glob, meta, _ = inputs.synthetic_inputs(n, 1234, (9, 13, 19), m.desc.num_input_channels,
                                                     m.desc.num_input_global_channels,
                                                     m.desc.num_input_meta_channels, rich=True)
    got = handle(name, prec, 64).forward(spatial, glob, meta)
    want = OracleNet(netgen.net_bytes(name)).forward(spatial, glob, meta)
    errs = max_err(got, want)
    assert max(errs.values()) <= TOL[prec], errs


@pytest.mark.parametrize("prec", [kc.PRECISION_F32, kc.PRECISION_F16])
def test_rows_are_independent(prec):
    """A row's outputs do not depend on its batch position or batch size (the reference's batch_buckets test)."""
    name = "tiny-nbt"
    spatial, glob, meta, _ = inputs.synthetic_inputs(40, 99, (9, 19), rich=True)
    h = handle(name, prec, 64)
    full = h.forward(spatial, glob)
    for i in (0, 17, 39):
        one = h.forward(spatial[i:i + 1], glob[i:i + 1])
        for k in KEYS:
            np.testing.assert_array_equal(one[k][0], full[k][i])


def test_b18_full_batch():
    """b18c384nbt at its benchmark batch (256 boards of 19x19, f16): every row against the float32 oracle (the
    batch spans 400 pair tiles of 256 PBL rows, the last one ragged), and the batch reversed gives every row
    bit-identical outputs (each row's arithmetic does not depend on which tile or CTA of the pair holds it)."""
    name = "b18c384nbt"
    spatial, glob, meta, _ = inputs.synthetic_inputs(256, 0xB200, (19,))
    h = handle(name, kc.PRECISION_F16, 256)
    got = h.forward(spatial, glob)
    for k in KEYS:
        assert np.all(np.isfinite(got[k])), k
    want = OracleNet(netgen.net_bytes(name)).forward(spatial, glob)
    errs = max_err(got, want)
    assert max(errs.values()) <= 2e-2, errs
    rev = h.forward(spatial[::-1].copy(), glob[::-1].copy())
    for k in KEYS:
        np.testing.assert_array_equal(rev[k][::-1], got[k])


def test_b18_mixed_boards():
    """The mixed-board configuration: b18c384nbt on 9x9 / 13x13 / 19x19 boards padded into 19x19 (masked BN,
    masked mean and -1e4 max pooling at the benchmark widths), batch 64, f16, every row against the float32
    oracle."""
    name = "b18c384nbt"
    spatial, glob, meta, sizes = inputs.synthetic_inputs(64, 0xB204, (9, 13, 19))
    assert set(sizes.tolist()) == {9, 13, 19}
    got = handle(name, kc.PRECISION_F16, 256).forward(spatial, glob)
    want = OracleNet(netgen.net_bytes(name)).forward(spatial, glob)
    errs = max_err(got, want)
    assert max(errs.values()) <= 2e-2, errs


def test_tf3_batch128():
    """tf3-b11c768 at its benchmark batch (128, bf16 tier): 12 heads of 64 at width 768, fixed-theta RoPE, spatial
    RMSNorm tip, 4 policy channels. Every output finite; 8 rows spread over the batch against the float32 oracle."""
    name = "tf3-b11c768"
    m = kc.Model(netgen.net_bytes(name))
    spatial, glob, meta, _ = inputs.synthetic_inputs(128, 0xB203, (19, 13, 9), m.desc.num_input_channels,
                                                     m.desc.num_input_global_channels)
    got = handle(name, kc.PRECISION_BF16, 128).forward(spatial, glob)
    for k in KEYS:
        assert np.all(np.isfinite(got[k])), k
    rows = [0, 1, 37, 63, 64, 100, 126, 127]
    want = OracleNet(netgen.net_bytes(name)).forward(spatial[rows], glob[rows])
    errs = {k: float(np.abs(got[k][rows] - want[k]).max()) for k in KEYS}
    assert max(errs.values()) <= 2e-2, errs
