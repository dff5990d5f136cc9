"""GPU test of the standalone gpool operator (kc_gpool_fc) against a float64 restatement of the reference graph's
gpool + matmul (tools/bin2onnx/bin2onnx.py gpool :1222-1230, matmul :1255)."""

import numpy as np
import pytest

from katago_cuda import api, inputs

pytestmark = pytest.mark.gpu


def gpool_reference(x, mask, w):
    """x [n,c,361] (masked), mask [n,361], w [3c,oc] -> [n,oc], float64."""
    x = x.astype(np.float64)
    m = mask.astype(np.float64)
    s = x.sum(axis=2)
    area = m.sum(axis=1, keepdims=True)
    mean = s / area
    scaled = mean * ((np.sqrt(area) - 14.0) * np.float64(np.float32(0.1)))
    mx = (x + (m[:, None, :] * 1e4 - 1e4)).max(axis=2)
    pooled = np.concatenate([mean, scaled, mx], axis=1)
    return pooled @ w.astype(np.float64)


def make_case(n, c, oc, seed):
    rng = np.random.default_rng(seed)
    spatial, _, _, _ = inputs.synthetic_inputs(n, seed, (9, 13, 19))
    mask = spatial[:, 0].reshape(n, 361)
    x = (rng.standard_normal((n, c, 361)) * mask[:, None, :]).astype(np.float32)
    w = (rng.standard_normal((3 * c, oc)) / np.sqrt(3 * c)).astype(np.float32)
    return x, mask.astype(np.float32), w


def run_op(fn, x, mask, w, reps=1):
    import torch
    dev = torch.device("cuda", 0)
    n, c, _ = x.shape
    oc = w.shape[1]
    dx, dm, dw = (torch.from_numpy(a).to(dev) for a in (x, mask, w))
    outs = []
    for _ in range(reps):
        dout = torch.full((n, oc), float("nan"), dtype=torch.float32, device=dev)
        fn(dx.data_ptr(), dm.data_ptr(), n, c, dw.data_ptr(), oc, dout.data_ptr(), 0)
        torch.cuda.synchronize()
        outs.append(dout.cpu().numpy())
    return outs


@pytest.mark.parametrize("n,c,oc", [(3, 16, 24), (37, 64, 128), (256, 96, 96)])
def test_gpool_fc_matches_reference(n, c, oc):
    x, mask, w = make_case(n, c, oc, 5 + n)
    (got,) = run_op(api.gpool_fc, x, mask, w)
    want = gpool_reference(x, mask, w)
    assert np.all(np.isfinite(got))
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)
