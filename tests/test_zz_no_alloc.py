"""kc_gpool_fc_noalloc — the gpool operator for callers that cannot allocate GPU memory (its scratch is a fixed
device array) — against the allocating kc_gpool_fc, through the C ABI, on two calls in a row. Collected last
(file name) so that a run stopping at the first failure has already run every other test; it also passes alone."""

import numpy as np
import pytest

from katago_cuda import api

from test_gpu_ops import gpool_reference, make_case, run_op

pytestmark = pytest.mark.gpu


def test_noalloc_matches_allocating_entry_point_twice():
    x, mask, w = make_case(37, 64, 128, 11)
    (ref,) = run_op(api.gpool_fc, x, mask, w)
    first, second = run_op(api.gpool_fc_noalloc, x, mask, w, reps=2)
    for got in (first, second):
        assert np.all(np.isfinite(got))
        np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(first, gpool_reference(x, mask, w), rtol=1e-4, atol=1e-4)


def test_noalloc_other_sizes_back_to_back():
    # a smaller call after a larger one: the shared scratch keeps stale data, which must not leak into the result
    for n, c, oc in [(256, 96, 96), (3, 16, 24)]:
        x, mask, w = make_case(n, c, oc, 3 + n)
        (ref,) = run_op(api.gpool_fc, x, mask, w)
        (got,) = run_op(api.gpool_fc_noalloc, x, mask, w)
        np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4)


def test_noalloc_rejects_oversized_scratch():
    n, c, oc = 1024, 128, 8  # n * 3c = 393216 > 262144
    assert n * 3 * c > api.GPOOL_NOALLOC_MAX_FLOATS
    x, mask, w = make_case(n, c, oc, 1)
    with pytest.raises(api.KcError) as e:
        run_op(api.gpool_fc_noalloc, x, mask, w)
    assert e.value.status == api.KC_ERR_INVALID
    assert "exceeds its fixed scratch" in str(e.value)
