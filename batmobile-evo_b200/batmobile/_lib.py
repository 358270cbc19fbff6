"""ctypes binding of libbatmobile_b200.so (declared in include/batmobile_b200.h).

The library is the only compute path: if it is missing this module raises at
import time; there is no CPU or PyTorch fallback.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libbatmobile_b200.so")

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_sz = ctypes.c_size_t
_f64 = ctypes.c_double
_f32 = ctypes.c_float
_bool = ctypes.c_bool

# name -> (restype, argtypes)
_SIGNATURES = {
    "bm_status_string": (ctypes.c_char_p, [_i32]),
    "bm_last_error": (ctypes.c_char_p, []),
    "bm_version": (_i32, []),
    "bm_launch_count": (_i64, []),
    "bm_probe_fp32": (_i32, [_p, _i32, _i32, _p]),
    "bm_probe_mma_tf32": (_i32, [_p, _i32, _i32, _p]),
    "bm_set_mix_precision": (_i32, [_i32]),
    "bm_get_mix_precision": (_i32, []),
    "bm_device_error_check": (_i32, []),
    "bm_selftest_wait_timeout": (_i32, [_p]),
    "bm_profile_start": (_i32, [_p]),
    "bm_profile_mark": (_i32, []),
    "bm_profile_stop": (_i32, []),
    "bm_profile_count": (_i32, []),
    "bm_profile_entry": (_i32, [_i32, ctypes.c_char_p, _i32, _p, _p]),
    "bm_tp_num_paths": (_i32, []),
    "bm_tp_path_info": (_i32, [_p]),
    "bm_sh_fwd": (_i32, [_p, _p, _i64, _i32, _p]),
    "bm_sh_bwd": (_i32, [_p, _p, _p, _i64, _i32, _p]),
    "bm_tp_simple_fwd": (_i32, [_p, _p, _p, _i64, _p]),
    "bm_tp_simple_bwd": (_i32, [_p, _p, _p, _p, _p, _i64, _p]),
    "bm_tp_fwd_workspace_bytes": (_sz, [_i64, _i32, _i32]),
    "bm_tp_fwd": (_i32, [_p, _p, _p, _p, _i64, _i32, _i32, _p, _sz, _p]),
    "bm_tp_fwd_noalloc_max_floats": (_sz, []),
    "bm_tp_fwd_noalloc": (_i32, [_p, _p, _p, _p, _i64, _i32, _i32, _p]),
    "bm_tp_bwd_workspace_bytes": (_sz, [_i64, _i32, _i32]),
    "bm_tp_bwd": (_i32, [_p, _p, _p, _p, _p, _p, _p, _i64, _i32, _i32, _p, _sz, _p]),
    "bm_csr_workspace_bytes": (_sz, [_i64, _i64]),
    "bm_edge_index_to_csr": (_i32, [_p, _p, _p, _i64, _i64, _p, _sz, _p]),
    "bm_csr_reverse": (_i32, [_p, _p, _i64, _i64, _p, _p]),
    "bm_fused_sh_tp_simple": (_i32, [_p, _p, _p, _p, _i64, _i64, _i32, _p]),
    "bm_fused_mp_simple": (_i32, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i32, _p]),
    "bm_fused_mp_weighted_workspace_bytes": (_sz, [_i64, _i32, _i32]),
    "bm_fused_mp_weighted": (_i32, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i32, _i32, _p, _sz, _p]),
    "bm_layer_fwd_workspace_bytes": (_sz, [_i64, _i64, _i32, _i32]),
    "bm_layer_fwd": (_i32, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i32, _i32, _p, _sz, _p]),
    "bm_layer_fwd_scaled": (_i32, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i32, _i32, _p, _sz, _p]),
    "bm_layer_bwd_scaled": (_i32, [_p] * 16 + [_i64, _i64, _i32, _i32, _p, _sz, _p]),
    "bm_layer_bwd_workspace_bytes": (_sz, [_i64, _i64, _i32, _i32]),
    "bm_layer_fwd_targets": (_i32, [_p] * 9 + [_i64, _i64, _i64, _i32, _i32, _p, _sz, _p]),
    "bm_layer_bwd_targets_workspace_bytes": (_sz, [_i64, _i64, _i64, _i32, _i32]),
    "bm_layer_bwd_targets": (_i32, [_p] * 16 + [_i64, _i64, _i64, _i32, _i32, _p, _sz, _p]),
    "bm_layer_bwd": (_i32, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                            _i64, _i64, _i32, _i32, _p, _sz, _p]),
    "bm_edge_grad_to_pos": (_i32, [_p, _p, _p, _p, _p, _p, _i64, _p]),
    "bm_nl_workspace_bytes": (_sz, [_i64, _p, _f64]),
    "bm_nl_count": (_i32, [_p, _i64, _p, _f64, _bool, _p, _p, _sz, _p]),
    "bm_nl_fill": (_i32, [_p, _i64, _p, _f64, _bool, _p, _i64, _p, _p, _p, _sz, _p]),
    "bm_nl_count_rows": (_i32, [_p, _i64, _i64, _p, _f64, _bool, _p, _p, _sz, _p]),
    "bm_nl_fill_rows": (_i32, [_p, _i64, _i64, _p, _f64, _bool, _p, _i64, _p, _p, _p, _sz, _p]),
    "bm_nl_workspace_bytes_cell": (_sz, [_i64, _p, _f64]),
    "bm_nl_count_cell": (_i32, [_p, _i64, _i64, _p, _f64, _bool, _p, _p, _sz, _p]),
    "bm_nl_fill_cell": (_i32, [_p, _i64, _i64, _p, _f64, _bool, _p, _i64, _p, _p, _p, _sz, _p]),
    "neighbor_list_cuda": (_i32, [_p, _p, _i64, _f32, _bool, _p, _p]),
    "neighbor_list_free": (None, [_p]),
    "neighbor_list_estimate_memory": (_sz, [_i64, _f32, _f32]),
}


class NeighborListResult(ctypes.Structure):
    """Layout of the reference's NeighborListResult (include/neighbor_list.cuh:25-33)."""
    _fields_ = [
        ("edge_index", ctypes.c_void_p),
        ("edge_vectors", ctypes.c_void_p),
        ("num_edges", ctypes.c_int64),
        ("d_edge_index", ctypes.c_void_p),
        ("d_edge_vectors", ctypes.c_void_p),
    ]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            "libbatmobile_b200.so not found at %s; build it with "
            "`python batmobile-evo_b200/build.py` (there is no CPU fallback)" % LIB_PATH)
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class BatmobileError(RuntimeError):
    pass


def check(status, what=""):
    if status != 0:
        msg = lib.bm_last_error().decode(errors="replace")
        kind = lib.bm_status_string(status).decode()
        raise BatmobileError("%s%s (%s)" % (what + ": " if what else "", msg, kind))


def exported_symbols():
    return list(_SIGNATURES)


def profile_report():
    """[(name, launches, total_ms)] of the last bm_profile_start/stop window."""
    out = []
    buf = ctypes.create_string_buffer(128)
    n = ctypes.c_int64()
    ms = ctypes.c_double()
    for i in range(lib.bm_profile_count()):
        check(lib.bm_profile_entry(i, buf, 128, ctypes.byref(n), ctypes.byref(ms)), "profile")
        out.append((buf.value.decode(), n.value, ms.value))
    return out
