"""Bit-packed inputs with the symmetry applied on the device (kc_enqueue_packed) and the reference's copy_outputs
run on the device, through the C ABI.

* For all 8 symmetries the network's raw outputs of packed rows with symmetry s are bit-identical to those of the
  float rows moved on the host by copy_with_symmetry (SymmetryHelpers::copy_inputs_with_symmetry,
  nninputs.rs:872), on the tensor-core (f16) and float32 stem paths and on mixed board sizes.
* The NNOutput rows (finish = 1) equal a numpy restatement of copy_outputs (backend.rs:622-731) applied to the raw
  rows, bit for bit (the optimism mix is rounded step by step on both sides).
* kc_get_output with a spatial value that is neither 0 nor 1 takes the float path (symmetry on the host) and
  agrees with the packed path's rows where the inputs are binary.
"""

import numpy as np
import pytest

import katago_cuda as kc
from katago_cuda import api, inputs, netgen

pytestmark = pytest.mark.gpu

KEYS = ("policy", "value", "scorevalue", "ownership")


def handle(name, prec, n):
    m = kc.Model(netgen.net_bytes(name))
    return m, kc.Handle(kc.Context(m, gpu_idxs=[0], precision=prec), max_batch=n, gpu_idx=0)


@pytest.mark.parametrize("name,prec", [("small-nbt", kc.PRECISION_F16), ("tiny-resnet", kc.PRECISION_F32),
                                       ("tiny-tf-learn", kc.PRECISION_BF16)])
def test_packed_rows_with_device_symmetry_match_host_symmetry(name, prec):
    n = 16
    m, h = handle(name, prec, n)
    d = m.desc
    spatial, glob, meta, _ = inputs.synthetic_inputs(n, 91, (9, 13, 19), d.num_input_channels,
                                                     d.num_input_global_channels, d.num_input_meta_channels,
                                                     rich=True)
    syms = np.arange(n, dtype=np.int32) % 8  # every symmetry, twice
    moved = np.stack([api.copy_with_symmetry(spatial[i:i + 1], 1, 19, 19, d.num_input_channels, int(syms[i]), False)[0]
                      for i in range(n)])
    want = h.forward(moved, glob, meta)
    got = h.forward_packed(spatial, glob, syms, meta)
    for k in KEYS:
        np.testing.assert_array_equal(got[k], want[k])
    # the symmetry matters: the identity gives other raw outputs on the transformed rows
    plain = h.forward_packed(spatial, glob, np.zeros(n, np.int32), meta)
    assert not np.array_equal(plain["policy"][1:], want["policy"][1:])


def copy_outputs(raw, sym, opt, P, version):
    """numpy restatement of copy_outputs (backend.rs:622-731) on one row's raw outputs."""
    pol = raw["policy"]
    o = np.float32(opt)
    if P == 2 or (P == 4 and version >= 16):
        mixed = (pol[0] + (pol[1] - pol[0]) * o).astype(np.float32)
    else:
        mixed = pol[0]
    inv = lambda plane: api.copy_with_symmetry(plane.reshape(1, 1, 19, 19), 1, 19, 19, 1, sym, True).reshape(-1)
    policy = np.concatenate([inv(mixed[:361]), mixed[361:]])
    sv = raw["scorevalue"]
    if version >= 9:
        misc = sv[:6]
    elif version >= 8:
        misc = np.array([sv[0], sv[1], sv[2], sv[3], 0, 0], np.float32)
    elif version >= 4:
        misc = np.array([sv[0], sv[1], sv[0], 0, 0, 0], np.float32)
    else:
        misc = np.array([sv[0], sv[0] * sv[0], sv[0], 0, 0, 0], np.float32)
    return policy, raw["value"], misc, inv(raw["ownership"][0])


@pytest.mark.parametrize("name", ["tiny-nbt", "tiny-resnet", "tiny-tf-learn", "tiny-v15-meta"])
def test_device_copy_outputs(name):
    n = 12
    m, h = handle(name, kc.PRECISION_F16, n)
    d = m.desc
    spatial, glob, meta, _ = inputs.synthetic_inputs(n, 17, (19, 13, 9), d.num_input_channels,
                                                     d.num_input_global_channels, d.num_input_meta_channels,
                                                     rich=True)
    rng = np.random.default_rng(9)
    syms = rng.integers(0, 8, size=n).astype(np.int32)
    opts = rng.choice([0.0, 0.25, 1.0], size=n).astype(np.float32)
    raw = h.forward_packed(spatial, glob, syms, meta)
    h.pk_opt[:n] = opts
    h.enqueue_packed(n, True)
    fin = np.array(h.wait_finished()[:n])
    for i in range(n):
        one = {k: raw[k][i] for k in KEYS}
        pol, val, misc, own = copy_outputs(one, int(syms[i]), opts[i], d.num_policy_channels, d.model_version)
        np.testing.assert_array_equal(fin[i, api.FINISHED_POLICY:api.FINISHED_POLICY + 362], pol)
        np.testing.assert_array_equal(fin[i, api.FINISHED_VALUE:api.FINISHED_VALUE + 3], val)
        np.testing.assert_array_equal(fin[i, api.FINISHED_MISC:api.FINISHED_MISC + 6], misc)
        np.testing.assert_array_equal(fin[i, api.FINISHED_OWNERSHIP:api.FINISHED_OWNERSHIP + 361], own)


def test_get_output_float_fallback_for_non_binary_planes():
    n = 6
    m, h = handle("tiny-nbt", kc.PRECISION_F32, n)
    spatial, glob, _, _ = inputs.synthetic_inputs(n, 5, (19, 9), rich=True)
    syms = [3, 5, 6, 7, 1, 2]
    opts = [0.0] * n
    packed = h.get_output([s.reshape(-1) for s in spatial], list(glob), None, syms, opts)
    odd = spatial.copy()
    odd[0, 7, 0, 0] = 0.5  # not a 0 / 1 feature: the whole batch goes as floats, row 0 differs
    floats = h.get_output([s.reshape(-1) for s in odd], list(glob), None, syms, opts)
    for k in ("policy", "value", "misc", "ownership"):
        np.testing.assert_array_equal(floats[k][1:], packed[k][1:])
    assert not np.array_equal(floats["policy"][0], packed["policy"][0])
