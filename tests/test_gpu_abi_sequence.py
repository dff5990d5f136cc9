"""The katago-nn-cuda Rust crate's call sequence through the C ABI, made by tests/abi_sequence.cpp (compiled here
with the system C++ compiler against libkatago_cuda.so): packed rows with the symmetry and copy_outputs on the
device, and the float fallback with the symmetry and copy_outputs on the host. Both must give kc_get_output's
NNOutput fields bit for bit (kc_get_output runs the same library paths in one call)."""

import os
import subprocess

import numpy as np
import pytest

import katago_cuda as kc
from katago_cuda import api, inputs, netgen

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def program(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("abi") / "abi_sequence")
    libdir = os.path.dirname(api.library_path())
    subprocess.check_call(["g++", "-std=c++17", "-O2", "-o", exe, os.path.join(HERE, "abi_sequence.cpp"),
                           "-L" + libdir, "-lkatago_cuda", "-Wl,-rpath," + libdir, "-lpthread"])
    return exe


@pytest.mark.parametrize("name,prec", [("tiny-nbt", kc.PRECISION_F16), ("tiny-tf-learn", kc.PRECISION_AUTO),
                                       ("tiny-resnet", kc.PRECISION_F32)])
@pytest.mark.parametrize("float_path", [0, 1])
def test_crate_call_sequence(program, tmp_path, name, prec, float_path):
    data = netgen.net_bytes(name)
    model_file = tmp_path / f"{name}.bin"
    model_file.write_bytes(data)
    m = kc.Model(data)
    d = m.desc
    n = 9
    spatial, glob, _, _ = inputs.synthetic_inputs(n, 44, (19, 13, 9), d.num_input_channels,
                                                  d.num_input_global_channels, rich=True)
    syms = (np.arange(n) * 5 % 8).astype(np.int32)
    opts = np.linspace(0, 1, n).astype(np.float32)
    with open(tmp_path / "in.bin", "wb") as f:
        f.write(np.array([n, d.num_input_channels, d.num_input_global_channels], np.int32).tobytes())
        for i in range(n):
            f.write(spatial[i].astype(np.float32).tobytes())
            f.write(glob[i].astype(np.float32).tobytes())
            f.write(np.int32(syms[i]).tobytes())
            f.write(np.float32(opts[i]).tobytes())
    subprocess.check_call([program, str(model_file), str(tmp_path / "in.bin"), str(tmp_path / "out.bin"),
                           str(prec), str(float_path)])
    got = np.fromfile(tmp_path / "out.bin", np.float32).reshape(n, api.FINISHED_ROW_LEN)
    h = kc.Handle(kc.Context(m, gpu_idxs=[0], precision=prec), max_batch=n, gpu_idx=0)
    want = h.get_output([s.reshape(-1) for s in spatial], list(glob), None, list(syms), list(opts))
    np.testing.assert_array_equal(got[:, api.FINISHED_POLICY:api.FINISHED_POLICY + 362], want["policy"])
    np.testing.assert_array_equal(got[:, api.FINISHED_VALUE:api.FINISHED_VALUE + 3], want["value"])
    np.testing.assert_array_equal(got[:, api.FINISHED_MISC:api.FINISHED_MISC + 6], want["misc"])
    np.testing.assert_array_equal(got[:, api.FINISHED_OWNERSHIP:api.FINISHED_OWNERSHIP + 361], want["ownership"])
