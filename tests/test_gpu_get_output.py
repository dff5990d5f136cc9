"""kc_get_output — the reference's whole get_output (crates/katago-nn-burn/src/backend.rs:410-731) — against the CPU
oracle plus a numpy restatement of its host logic: each row's inputs copied with its symmetry, raw outputs, policy
optimism mix for 2-channel (or v16+ 4-channel) policies, inverse symmetry on policy and ownership, score fields by
model version."""

import numpy as np
import pytest

import katago_cuda as kc
from katago_cuda import inputs, netgen
from oracle.oracle import OracleNet

pytestmark = pytest.mark.gpu


def sym_loc(x, y, size, s):
    # getSymLoc (nninputs.rs:909-924): flipX (bit 1), flipY (bit 0), then transpose (bit 2)
    if s & 2:
        x = size - x - 1
    if s & 1:
        y = size - y - 1
    if s & 4:
        x, y = y, x
    return x, y


def apply_sym(planes, s):
    """planes [C,19,19] in board space -> net space: dst[sy, sx] = src[y, x]."""
    out = np.empty_like(planes)
    for y in range(19):
        for x in range(19):
            sx, sy = sym_loc(x, y, 19, s)
            out[:, sy, sx] = planes[:, y, x]
    return out


def undo_sym(plane, s):
    """net-space [19,19] -> board space: out[y, x] = net[sy, sx]."""
    out = np.empty_like(plane)
    for y in range(19):
        for x in range(19):
            sx, sy = sym_loc(x, y, 19, s)
            out[y, x] = plane[sy, sx]
    return out


@pytest.mark.parametrize("name", ["tiny-resnet", "tiny-nbt", "tiny-tf-learn", "tiny-v15-meta"])
def test_get_output_matches_reference_logic(name):
    data = netgen.net_bytes(name)
    model = kc.Model(data)
    d = model.desc
    n = 8
    spatial, glob, meta, _ = inputs.synthetic_inputs(n, 77, (19, 13, 9), d.num_input_channels,
                                                     d.num_input_global_channels, d.num_input_meta_channels,
                                                     rich=True)
    rng = np.random.default_rng(5)
    syms = [int(s) for s in rng.integers(0, 8, size=n)]
    opts = [float(o) for o in rng.choice([0.0, 0.5, 1.0], size=n)]
    h = kc.Handle(kc.Context(model, [0], kc.PRECISION_F32), max_batch=n, gpu_idx=0)
    got = h.get_output([spatial[i].reshape(-1) for i in range(n)], [glob[i] for i in range(n)],
                       [meta[i] for i in range(n)] if d.num_input_meta_channels else None, syms, opts)

    sym_in = np.stack([apply_sym(spatial[i], syms[i]) for i in range(n)])
    raw = OracleNet(data).forward(sym_in, glob, meta)
    P, v = d.num_policy_channels, d.model_version
    for i in range(n):
        pol = raw["policy"][i]
        if P == 2 or (P == 4 and v >= 16):
            mixed = pol[0] + (pol[1] - pol[0]) * np.float32(opts[i])
        else:
            mixed = pol[0]
        want_pol = np.concatenate([undo_sym(mixed[:361].reshape(19, 19), syms[i]).reshape(-1), mixed[361:]])
        np.testing.assert_allclose(got["policy"][i], want_pol, atol=1e-4, rtol=0)
        np.testing.assert_allclose(got["value"][i], raw["value"][i], atol=1e-4, rtol=0)
        own = undo_sym(raw["ownership"][i, 0], syms[i]).reshape(-1)
        np.testing.assert_allclose(got["ownership"][i], own, atol=1e-4, rtol=0)
        sv = raw["scorevalue"][i]
        want_misc = list(sv[:6]) if v >= 9 else [sv[0], sv[1], sv[2], sv[3], 0.0, 0.0]
        np.testing.assert_allclose(got["misc"][i], np.array(want_misc, np.float32), atol=1e-4, rtol=0)


def test_get_output_rejects_bad_sizes():
    model = kc.Model(netgen.net_bytes("tiny-resnet"))
    h = kc.Handle(kc.Context(model, [0], kc.PRECISION_F32), max_batch=2, gpu_idx=0)
    spatial, glob, _, _ = inputs.synthetic_inputs(3, 1, (19,))
    with pytest.raises(kc.KcError) as e:
        h.get_output([s.reshape(-1) for s in spatial], list(glob), None, [0, 0, 0], [0.0, 0.0, 0.0])
    assert e.value.status == kc.api.KC_ERR_INVALID
