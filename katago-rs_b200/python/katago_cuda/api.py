"""ctypes binding of libkatago_cuda.so.

Mirrors the reference backend's NeuralNet steps (crates/katago-nn-burn/src/backend.rs): Model.load ~
load_model_file, Context ~ create_compute_context, Handle ~ create_compute_handle + create_input_buffers,
Handle.get_output ~ get_output, and the asynchronous halves Handle.enqueue / Handle.wait of run_network.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(os.path.dirname(HERE))  # katago-rs_b200/
HEADER = os.path.join(os.path.dirname(PKG), "include", "katago_cuda.h")

PRECISION_F32, PRECISION_F16, PRECISION_BF16, PRECISION_AUTO = 0, 1, 2, 3
KC_OK, KC_ERR_INVALID, KC_ERR_PARSE, KC_ERR_CUDA, KC_ERR_TIMEOUT, KC_ERR_DEVICE, KC_ERR_NO_DEVICE = range(7)

_LIB = None


def library_path() -> str:
    return os.environ.get("KATAGO_CUDA_LIB", os.path.join(PKG, "lib", "libkatago_cuda.so"))


class KcError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status = status


class Desc(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char * 128),
        ("model_version", ctypes.c_int32),
        ("num_input_channels", ctypes.c_int32),
        ("num_input_global_channels", ctypes.c_int32),
        ("num_input_meta_channels", ctypes.c_int32),
        ("meta_encoder_version", ctypes.c_int32),
        ("num_policy_channels", ctypes.c_int32),
        ("num_value_channels", ctypes.c_int32),
        ("num_score_value_channels", ctypes.c_int32),
        ("num_ownership_channels", ctypes.c_int32),
        ("trunk_num_blocks", ctypes.c_int32),
        ("trunk_num_channels", ctypes.c_int32),
        ("trunk_norm_kind", ctypes.c_int32),
        ("has_any_transformer_blocks", ctypes.c_int32),
        ("has_any_nested_bottleneck_blocks", ctypes.c_int32),
        ("post_process_from_header", ctypes.c_int32),
        ("prefer_pass_alive_under_suicide_rules", ctypes.c_int32),
        ("prefer_exclude_territory_adjacent_to_atari", ctypes.c_int32),
        ("num_parameters", ctypes.c_int64),
        ("trunk_spatial_conv_depth", ctypes.c_double),
        ("post_process", ctypes.c_float * 8),
    ]


P = ctypes.c_void_p
I = ctypes.c_int
FP = ctypes.POINTER(ctypes.c_float)
FPP = ctypes.POINTER(FP)

_SIGS = {
    "kc_last_error": ([], ctypes.c_char_p),
    "kc_device_count": ([ctypes.POINTER(I)], I),
    "kc_model_load": ([ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.POINTER(P)], I),
    "kc_model_desc": ([P, ctypes.POINTER(Desc)], I),
    "kc_model_destroy": ([P], I),
    "kc_model_flops": ([P, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)], I),
    "kc_context_create": ([ctypes.POINTER(I), I, I, I, I, P, ctypes.POINTER(P)], I),
    "kc_context_precision": ([P, ctypes.POINTER(I)], I),
    "kc_context_destroy": ([P], I),
    "kc_handle_create": ([P, I, I, I, ctypes.POINTER(P)], I),
    "kc_handle_destroy": ([P], I),
    "kc_handle_input_ptrs": ([P, FPP, FPP, FPP], I),
    "kc_handle_output_layout": ([P] + [ctypes.POINTER(I)] * 5, I),
    "kc_enqueue": ([P, I], I),
    "kc_wait": ([P, I, FPP], I),
    "kc_enqueue_device": ([P, I, P, P, P, P], I),
    "kc_synchronize": ([P, I], I),
    "kc_handle_stream": ([P, ctypes.POINTER(P)], I),
    "kc_get_output": ([P, I, FPP, FPP, FPP, ctypes.POINTER(I), FP, I, FP, FP, FP, FP], I),
    "kc_handle_set_profiling": ([P, I], I),
    "kc_handle_profile": ([P, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64), I], I),
    "kc_handle_launch_count": ([P, I, ctypes.POINTER(I)], I),
    "kc_copy_with_symmetry": ([FP, FP, I, I, I, I, I, I], I),
    "kc_gpool_fc": ([P, P, I, I, P, I, P, P], I),
    "kc_gpool_fc_noalloc": ([P, P, I, I, P, I, P, P], I),
    "kc_selftest_device_timeout": ([P, I], I),
    "kc_handle_packed_input_ptrs": ([P, ctypes.POINTER(ctypes.POINTER(ctypes.c_uint32)), FPP, FPP,
                                     ctypes.POINTER(ctypes.POINTER(ctypes.c_int32)), FPP], I),
    "kc_enqueue_packed": ([P, I, I], I),
    "kc_pack_spatial": ([FP, I, ctypes.POINTER(ctypes.c_uint32)], I),
    "kc_symmetry_table": ([I, I, ctypes.POINTER(I)], I),
}
PACKED_WORDS_PER_PLANE = 12
FINISHED_ROW_LEN, FINISHED_POLICY, FINISHED_VALUE, FINISHED_MISC, FINISHED_OWNERSHIP = 732, 0, 362, 365, 371
GPOOL_NOALLOC_MAX_FLOATS = 262144


def lib():
    """The loaded library. Raises if it was not built (no fallback)."""
    global _LIB
    if _LIB is None:
        path = library_path()
        if not os.path.exists(path):
            raise RuntimeError(f"libkatago_cuda.so not found at {path}: build it with `make -C katago-rs_b200` "
                               f"(or __graft_entry__.build())")
        L = ctypes.CDLL(path)
        for name, (args, res) in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _LIB = L
    return _LIB


def _check(rc: int):
    if rc != KC_OK:
        raise KcError(rc, lib().kc_last_error().decode(errors="replace"))


def _fp(a: np.ndarray):
    return a.ctypes.data_as(FP)


def device_count() -> int:
    c = I(0)
    _check(lib().kc_device_count(ctypes.byref(c)))
    return c.value


class Model:
    """A parsed model file (NeuralNet::load_model_file). No device is used."""

    def __init__(self, data: bytes, file_name: Optional[str] = "model.bin"):
        h = P()
        _check(lib().kc_model_load(data, len(data), file_name.encode() if file_name else None, ctypes.byref(h)))
        self.h = h
        d = Desc()
        _check(lib().kc_model_desc(self.h, ctypes.byref(d)))
        self.desc = d

    def flops(self):
        t, c3 = ctypes.c_double(), ctypes.c_double()
        _check(lib().kc_model_flops(self.h, ctypes.byref(t), ctypes.byref(c3)))
        return t.value, c3.value

    def close(self):
        if getattr(self, "h", None):
            lib().kc_model_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()


class Context:
    """NeuralNet::create_compute_context."""

    def __init__(self, model: Model, gpu_idxs: Sequence[int] = (-1,), precision: int = PRECISION_AUTO,
                 nn_x_len: int = 19, nn_y_len: int = 19):
        arr = (I * len(gpu_idxs))(*gpu_idxs)
        h = P()
        _check(lib().kc_context_create(arr, len(gpu_idxs), nn_x_len, nn_y_len, precision, model.h, ctypes.byref(h)))
        self.h = h
        self.model = model
        p = I()
        _check(lib().kc_context_precision(self.h, ctypes.byref(p)))
        self.precision = p.value

    def close(self):
        if getattr(self, "h", None):
            lib().kc_context_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()


class Handle:
    """NeuralNet::create_compute_handle plus its pinned input buffers."""

    def __init__(self, ctx: Context, max_batch: int, gpu_idx: int = -1):
        h = P()
        _check(lib().kc_handle_create(ctx.h, gpu_idx, max_batch, 0, ctypes.byref(h)))
        self.h = h
        self.ctx = ctx
        self.max_batch = max_batch
        d = ctx.model.desc
        self.n_spatial = d.num_input_channels * 361
        self.n_global = d.num_input_global_channels
        self.n_meta = d.num_input_meta_channels
        s, g, m = FP(), FP(), FP()
        _check(lib().kc_handle_input_ptrs(self.h, ctypes.byref(s), ctypes.byref(g), ctypes.byref(m)))
        self.spatial = np.ctypeslib.as_array(s, shape=(max_batch, d.num_input_channels, 19, 19))
        self.glob = np.ctypeslib.as_array(g, shape=(max_batch, self.n_global))
        self.meta = np.ctypeslib.as_array(m, shape=(max_batch, self.n_meta)) if self.n_meta else None
        vals = [I() for _ in range(5)]
        _check(lib().kc_handle_output_layout(self.h, *[ctypes.byref(v) for v in vals]))
        self.row_len, self.policy_off, self.value_off, self.score_off, self.own_off = [v.value for v in vals]
        self.P = d.num_policy_channels
        b, g, m, sy, op = (ctypes.POINTER(ctypes.c_uint32)(), FP(), FP(), ctypes.POINTER(ctypes.c_int32)(), FP())
        _check(lib().kc_handle_packed_input_ptrs(self.h, ctypes.byref(b), ctypes.byref(g), ctypes.byref(m),
                                                 ctypes.byref(sy), ctypes.byref(op)))
        self.pk_bits = np.ctypeslib.as_array(b, shape=(max_batch, d.num_input_channels, PACKED_WORDS_PER_PLANE))
        self.pk_glob = np.ctypeslib.as_array(g, shape=(max_batch, self.n_global))
        self.pk_meta = np.ctypeslib.as_array(m, shape=(max_batch, self.n_meta)) if self.n_meta else None
        self.pk_sym = np.ctypeslib.as_array(sy, shape=(max_batch,))
        self.pk_opt = np.ctypeslib.as_array(op, shape=(max_batch,))

    def close(self):
        if getattr(self, "h", None):
            lib().kc_handle_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    # ---- raw forward --------------------------------------------------------------------------------------------
    def enqueue(self, n: int):
        _check(lib().kc_enqueue(self.h, n))

    def wait(self, timeout_ms: int = -1) -> np.ndarray:
        """The n output rows of the last enqueue (a view of pinned memory, valid until the next enqueue)."""
        p = FP()
        _check(lib().kc_wait(self.h, timeout_ms, ctypes.byref(p)))
        return np.ctypeslib.as_array(p, shape=(self.max_batch, self.row_len))

    def forward(self, spatial, glob, meta=None, timeout_ms: int = 120000) -> dict:
        """Raw outputs of the reference graph for n rows: policy [n,P,362], value [n,3], scorevalue [n,Sv],
        ownership [n,1,19,19]."""
        n = spatial.shape[0]
        self.spatial[:n] = spatial
        self.glob[:n] = glob
        if self.n_meta:
            self.meta[:n] = meta
        self.enqueue(n)
        rows = np.array(self.wait(timeout_ms)[:n])
        return self.split(rows)

    def split(self, rows: np.ndarray) -> dict:
        n = rows.shape[0]
        return {
            "policy": rows[:, self.policy_off:self.policy_off + self.P * 362].reshape(n, self.P, 362),
            "value": rows[:, self.value_off:self.value_off + 3],
            "scorevalue": rows[:, self.score_off:self.own_off],
            "ownership": rows[:, self.own_off:self.own_off + 361].reshape(n, 1, 19, 19),
        }

    def enqueue_packed(self, n: int, finish: bool):
        """kc_enqueue_packed: rows [0, n) of the packed staging (pk_bits, pk_glob, pk_meta, pk_sym, pk_opt)."""
        _check(lib().kc_enqueue_packed(self.h, n, int(finish)))

    def wait_finished(self, timeout_ms: int = -1) -> np.ndarray:
        """The NNOutput rows [max_batch, FINISHED_ROW_LEN] of the last kc_enqueue_packed(finish=1)."""
        p = FP()
        _check(lib().kc_wait(self.h, timeout_ms, ctypes.byref(p)))
        return np.ctypeslib.as_array(p, shape=(self.max_batch, FINISHED_ROW_LEN))

    def forward_packed(self, spatial, glob, symmetry, meta=None, timeout_ms: int = 120000) -> dict:
        """Raw outputs (as forward) of n rows sent bit-packed with per-row symmetries applied on the device."""
        n = spatial.shape[0]
        for i in range(n):
            self.pk_bits[i] = pack_spatial(spatial[i])
        self.pk_glob[:n] = glob
        if self.n_meta:
            self.pk_meta[:n] = meta
        self.pk_sym[:n] = symmetry
        self.enqueue_packed(n, False)
        rows = np.array(self.wait(timeout_ms)[:n])
        return self.split(rows)

    def enqueue_device(self, n: int, d_spatial: int, d_global: int, d_meta: int, d_out: int):
        _check(lib().kc_enqueue_device(self.h, n, d_spatial, d_global, d_meta or None, d_out))

    def stream_ptr(self) -> int:
        s = P()
        _check(lib().kc_handle_stream(self.h, ctypes.byref(s)))
        return s.value or 0

    def synchronize(self, timeout_ms: int = -1):
        _check(lib().kc_synchronize(self.h, timeout_ms))

    def selftest_device_timeout(self, limit_us: int):
        """kc_selftest_device_timeout: enqueue a kernel whose bounded wait runs out after `limit_us`."""
        _check(lib().kc_selftest_device_timeout(self.h, limit_us))

    # ---- NeuralNet::get_output --------------------------------------------------------------------------------
    def get_output(self, spatial_rows, global_rows, meta_rows, symmetry, policy_optimism, want_ownership=True,
                   timeout_ms: int = 120000) -> dict:
        n = len(spatial_rows)
        sp = [np.ascontiguousarray(r, np.float32) for r in spatial_rows]
        gl = [np.ascontiguousarray(r, np.float32) for r in global_rows]
        sp_arr = (FP * n)(*[_fp(r) for r in sp])
        gl_arr = (FP * n)(*[_fp(r) for r in gl])
        me_arr = None
        if self.n_meta:
            me = [np.ascontiguousarray(r, np.float32) for r in meta_rows]
            me_arr = (FP * n)(*[_fp(r) for r in me])
        sym = (I * n)(*[int(s) for s in symmetry])
        opt = np.ascontiguousarray(policy_optimism, np.float32)
        pol = np.zeros((n, 362), np.float32)
        val = np.zeros((n, 3), np.float32)
        misc = np.zeros((n, 6), np.float32)
        own = np.zeros((n, 361), np.float32) if want_ownership else None
        _check(lib().kc_get_output(self.h, n, sp_arr, gl_arr, me_arr, sym, _fp(opt), timeout_ms, _fp(pol), _fp(val),
                                   _fp(misc), _fp(own) if own is not None else None))
        return {"policy": pol, "value": val, "misc": misc, "ownership": own}

    # ---- measurement ------------------------------------------------------------------------------------------
    def set_profiling(self, on: bool):
        _check(lib().kc_handle_set_profiling(self.h, int(on)))

    def profile(self):
        ms = (ctypes.c_double * 5)()
        n = (ctypes.c_int64 * 5)()
        _check(lib().kc_handle_profile(self.h, ms, n, 5))
        names = ["conv3x3", "linear", "stem", "attention", "other"]
        return {k: (ms[i], n[i]) for i, k in enumerate(names)}

    def launch_count(self, n: int) -> int:
        c = I()
        _check(lib().kc_handle_launch_count(self.h, n, ctypes.byref(c)))
        return c.value


def gpool_fc(d_x: int, d_mask: int, n: int, c: int, d_w: int, oc: int, d_out: int, stream: int = 0):
    """kc_gpool_fc on device pointers (masked global pooling + gpool-to-bias matmul)."""
    _check(lib().kc_gpool_fc(d_x, d_mask, n, c, d_w, oc, d_out, stream or None))


def gpool_fc_noalloc(d_x: int, d_mask: int, n: int, c: int, d_w: int, oc: int, d_out: int, stream: int = 0):
    """kc_gpool_fc_noalloc: the same operator with its scratch in a fixed device array (no allocation)."""
    _check(lib().kc_gpool_fc_noalloc(d_x, d_mask, n, c, d_w, oc, d_out, stream or None))


def pack_spatial(planes: np.ndarray) -> np.ndarray:
    """kc_pack_spatial: float planes [C, 19, 19] of 0 / 1 -> [C, PACKED_WORDS_PER_PLANE] uint32."""
    planes = np.ascontiguousarray(planes, np.float32)
    c = planes.shape[0]
    out = np.zeros((c, PACKED_WORDS_PER_PLANE), np.uint32)
    _check(lib().kc_pack_spatial(_fp(planes), c, out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))))
    return out


def symmetry_table(symmetry: int, reverse: bool) -> np.ndarray:
    t = np.zeros(361, np.int32)
    _check(lib().kc_symmetry_table(symmetry, int(reverse), t.ctypes.data_as(ctypes.POINTER(I))))
    return t


def copy_with_symmetry(src: np.ndarray, n: int, h: int, w: int, c: int, symmetry: int, reverse: bool) -> np.ndarray:
    src = np.ascontiguousarray(src, np.float32)
    dst = np.zeros_like(src)
    _check(lib().kc_copy_with_symmetry(_fp(src), _fp(dst), n, h, w, c, symmetry, int(reverse)))
    return dst
