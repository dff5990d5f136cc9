"""Host-side symmetry helpers (the reference's SymmetryHelpers, crates/katago-core/src/neuralnet/nninputs.rs:756-899)
exported by the library: a numpy restatement of getSymLoc semantics and the inverse property. CPU only."""

import numpy as np
import pytest

from katago_cuda import api


def sym_loc(x, y, size, s):
    # nninputs.rs:909-924: flipX (bit 1), flipY (bit 0), then transpose (bit 2)
    if s & 2:
        x = size - x - 1
    if s & 1:
        y = size - y - 1
    if s & 4:
        x, y = y, x
    return x, y


@pytest.mark.parametrize("s", range(8))
def test_inputs_follow_getsymloc(s):
    rng = np.random.default_rng(s)
    src = rng.standard_normal((1, 3, 19, 19)).astype(np.float32)
    dst = api.copy_with_symmetry(src, 1, 19, 19, 3, s, False)
    for y in range(19):
        for x in range(19):
            sx, sy = sym_loc(x, y, 19, s)
            np.testing.assert_array_equal(dst[0, :, sy, sx], src[0, :, y, x])


@pytest.mark.parametrize("s", range(8))
def test_outputs_invert_inputs(s):
    rng = np.random.default_rng(100 + s)
    src = rng.standard_normal((1, 1, 19, 19)).astype(np.float32)
    fwd = api.copy_with_symmetry(src, 1, 19, 19, 1, s, False)
    back = api.copy_with_symmetry(fwd, 1, 19, 19, 1, s, True)
    np.testing.assert_array_equal(back, src)


@pytest.mark.parametrize("s", range(8))
def test_device_symmetry_tables_match_host_copies(s):
    """The point mappings the GPU applies (input planes as they are read, outputs as they are written back) are the
    moves of the host copy_with_symmetry."""
    src = np.arange(361, dtype=np.float32).reshape(1, 1, 19, 19)
    fwd = api.copy_with_symmetry(src, 1, 19, 19, 1, s, False).reshape(-1)
    np.testing.assert_array_equal(api.symmetry_table(s, False), fwd.astype(np.int32))
    rev = api.copy_with_symmetry(src, 1, 19, 19, 1, s, True).reshape(-1)
    table = api.symmetry_table(s, True)
    np.testing.assert_array_equal(rev[table], np.arange(361, dtype=np.float32))


def test_pack_spatial_bits():
    rng = np.random.default_rng(3)
    planes = (rng.random((22, 19, 19)) < 0.3).astype(np.float32)
    bits = api.pack_spatial(planes)
    assert bits.shape == (22, api.PACKED_WORDS_PER_PLANE)
    flat = planes.reshape(22, 361)
    for c in range(22):
        for p in range(384):
            bit = (int(bits[c, p // 32]) >> (p % 32)) & 1
            assert bit == (int(flat[c, p]) if p < 361 else 0)


def test_pack_spatial_rejects_non_binary():
    planes = np.zeros((22, 19, 19), np.float32)
    planes[5, 3, 4] = 0.5
    with pytest.raises(api.KcError) as e:
        api.pack_spatial(planes)
    assert e.value.status == api.KC_ERR_INVALID
