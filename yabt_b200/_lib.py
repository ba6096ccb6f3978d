"""ctypes binding of libyabt_b200.so (the C ABI declared in include/yabt_b200.h).

The library is built in-tree by ``yabt_b200.build``. There is no fallback:
if the shared library is missing or a CUDA device is absent, calls raise.
Loading is guarded by a lock, as the reference guards its C grower loader
(yabt/grow_c.py:49,215).
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
# YABT_LIB_VARIANT=checked loads the bounds-checked build (python -m yabt_b200.build --bounds-check)
LIB_PATH = os.path.join(_HERE, "libyabt_b200_checked.so" if os.environ.get("YABT_LIB_VARIANT") == "checked"
                        else "libyabt_b200.so")
_LOCK = threading.Lock()
_LIB = None

c_ll = ctypes.c_longlong
c_int = ctypes.c_int
c_float = ctypes.c_float
c_vp = ctypes.c_void_p


class TreeArgs(ctypes.Structure):
    """Mirror of ``yabt_tree_args`` (include/yabt_b200.h)."""
    _fields_ = [
        ("bins", c_vp), ("grad", c_vp), ("hess", c_vp), ("edges", c_vp), ("edge_off", c_vp),
        ("edge_cnt", c_vp), ("scales", c_vp), ("feature_mask", c_vp), ("interaction", c_vp),
        ("reg_lambda", c_float), ("gamma", c_float), ("min_child_weight", c_float),
        ("learning_rate", c_float), ("interaction_boost", c_float), ("min_samples_leaf", ctypes.c_int32),
        ("feature", c_vp), ("threshold", c_vp), ("left", c_vp), ("right", c_vp), ("value", c_vp),
        ("gate_scale", c_vp), ("leaf_of_row", c_vp), ("meta", c_vp), ("bins_fm", c_vp),
        ("root_rows", c_vp), ("n_root", c_ll),
    ]


class LeafNetArgs(ctypes.Structure):
    """Mirror of ``yabt_leafnet_args``."""
    _fields_ = [
        ("feature", c_vp), ("value", c_vp), ("max_nodes", ctypes.c_int32), ("meta", c_vp),
        ("leaf_src", c_vp), ("leaf_begin", c_vp), ("leaf_count", c_vp), ("fin", c_vp),
        ("list0", c_vp), ("list1", c_vp), ("leaf_of_row", c_vp), ("Xfm", c_vp), ("col_mean", c_vp),
        ("col_std", c_vp), ("margin", c_vp), ("y", c_vp), ("n", c_ll), ("F", ctypes.c_int32),
        ("K", ctypes.c_int32), ("loss", ctypes.c_int32), ("min_samples", ctypes.c_int32),
        ("l2", c_float), ("learning_rate", c_float), ("feats", c_vp), ("linear", c_vp),
        ("lo", c_vp), ("hi", c_vp), ("has_nets", c_vp),
    ]


class UpdateArgs(ctypes.Structure):
    """Mirror of ``yabt_update_args``."""
    _fields_ = [
        ("leaf_of_row", c_vp), ("max_nodes", ctypes.c_int32), ("value", c_vp), ("linear", c_vp),
        ("lo", c_vp), ("hi", c_vp), ("feats", c_vp), ("has_nets", c_vp), ("K", ctypes.c_int32),
        ("Xfm", c_vp), ("n", c_ll),
        ("margin", c_vp), ("y", c_vp), ("grad", c_vp), ("hess", c_vp), ("loss", ctypes.c_int32),
    ]


# (name, restype, argtypes) of every exported symbol
SIGNATURES = [
    ("yabt_version", c_int, []),
    ("yabt_last_error", c_int, [ctypes.c_char_p, c_int]),
    ("yabt_launch_count", c_ll, []),
    ("yabt_launch_count_device", c_ll, []),
    ("yabt_launch_count_device_reset", c_int, [c_vp]),
    ("yabt_probe_shared_red", c_int, [c_int, c_int, c_vp, c_vp, ctypes.POINTER(ctypes.c_float),
                                      ctypes.POINTER(ctypes.c_longlong)]),
    ("yabt_probe_shared_red_masked", c_int, [c_int, c_int, c_int, c_vp, c_vp, ctypes.POINTER(ctypes.c_float),
                                             ctypes.POINTER(ctypes.c_longlong)]),
    ("yabt_phase_count", c_int, []),
    ("yabt_phase_name", c_int, [c_int, ctypes.c_char_p, c_int]),
    ("yabt_phase_timing", c_int, [c_int]),
    ("yabt_phase_read", c_int, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(c_ll), c_int]),
    ("yabt_phase_push", c_int, [c_int, c_vp]),
    ("yabt_phase_pop", c_int, []),
    ("yabt_grower_set_timing", c_int, [c_vp, c_int]),
    ("yabt_grower_hist_times", c_int, [c_vp, ctypes.POINTER(c_float), c_int, ctypes.POINTER(c_int)]),
    ("yabt_grower_hist_rows", c_int, [c_vp, ctypes.POINTER(c_ll), c_int]),
    ("yabt_grower_acc_reset", c_int, [c_vp, c_vp]),
    ("yabt_grower_acc_read", c_int, [c_vp, ctypes.POINTER(c_ll)]),
    ("yabt_bin_matrix_bytes", c_ll, [c_ll, c_int]),
    ("yabt_bin_address", c_int, [c_ll, c_int, c_int, ctypes.POINTER(c_ll), ctypes.POINTER(c_int),
                                 ctypes.POINTER(c_int)]),
    ("yabt_pack_bins", c_int, [c_vp, c_ll, c_int, c_vp, c_vp]),
    ("yabt_grower_create", c_int, [c_ll, c_int, c_int, c_int, c_int, ctypes.POINTER(c_vp)]),
    ("yabt_grower_workspace_bytes", c_ll, [c_vp]),
    ("yabt_grower_bind", c_int, [c_vp, c_vp, c_ll, c_vp]),
    ("yabt_grower_destroy", c_int, [c_vp]),
    ("yabt_grower_max_nodes", c_int, [c_vp]),
    ("yabt_grower_levels", c_int, [c_vp]),
    ("yabt_grow_tree", c_int, [c_vp, ctypes.POINTER(TreeArgs), c_vp]),
    ("yabt_grow_tree_bestfirst", c_int, [c_vp, ctypes.POINTER(TreeArgs), c_vp]),
    ("yabt_grower_set_bestfirst_f64", c_int, [c_vp, c_int]),
    ("yabt_grower_set_root_count_cache", c_int, [c_vp, c_int]),
    ("yabt_grower_root_counts", c_int, [c_vp, c_vp, c_vp]),
    ("yabt_mt_workspace_bytes", c_ll, [c_vp, c_int]),
    ("yabt_grow_tree_multitask", c_int, [c_vp, ctypes.POINTER(TreeArgs), c_int, c_vp, c_vp, c_ll, c_vp, c_vp]),
    ("yabt_mt_update", c_int, [c_vp, c_vp, c_int, c_ll, c_vp, c_vp, c_vp, c_vp]),
    ("yabt_grow_bf_root_hist", c_int, [c_vp, ctypes.POINTER(TreeArgs), c_vp]),
    ("yabt_grow_bf_split", c_int, [c_vp, ctypes.POINTER(TreeArgs), c_int, c_vp]),
    ("yabt_grow_bf_scan", c_int, [c_vp, ctypes.POINTER(TreeArgs), c_int, c_vp]),
    ("yabt_grow_begin", c_int, [c_vp, ctypes.POINTER(TreeArgs), c_vp]),
    ("yabt_grow_init", c_int, [c_vp, ctypes.POINTER(TreeArgs), c_vp]),
    ("yabt_grow_hist", c_int, [c_vp, ctypes.POINTER(TreeArgs), c_int, c_vp]),
    ("yabt_grow_split", c_int, [c_vp, ctypes.POINTER(TreeArgs), c_int, c_vp]),
    ("yabt_grow_end", c_int, [c_vp, ctypes.POINTER(TreeArgs), c_vp]),
    ("yabt_grow_amax_ptr", c_vp, [c_vp]),
    ("yabt_grow_small_ptr", c_vp, [c_vp]),
    ("yabt_grow_level_ptr", c_vp, [c_vp]),
    ("yabt_grower_set_level_wait", c_int, [c_vp, c_int]),
    ("yabt_grower_set_level_loop", c_int, [c_vp, c_int]),
    ("yabt_grower_level_loop_start", c_int, [c_vp]),
    ("yabt_grow_apply_all", c_int, [c_vp, ctypes.POINTER(TreeArgs), c_vp]),
    ("yabt_group_rows_workspace_bytes", c_ll, [c_ll, c_int]),
    ("yabt_group_rows", c_int, [c_vp, c_ll, c_int, c_vp, c_ll, c_vp, c_vp, c_vp, c_vp]),
    ("yabt_xchg_header_bytes", c_ll, []),
    ("yabt_xchg_alloc", c_int, [c_ll, ctypes.POINTER(c_vp), c_vp]),
    ("yabt_xchg_open", c_int, [c_vp, ctypes.POINTER(c_vp)]),
    ("yabt_xchg_close", c_int, [c_vp]),
    ("yabt_xchg_free", c_int, [c_vp]),
    ("yabt_grower_set_small", c_int, [c_vp, c_vp, c_ll]),
    ("yabt_grow_xreduce", c_int, [c_vp, ctypes.POINTER(c_vp), c_int, c_int, c_int, ctypes.c_uint, c_vp]),
    ("yabt_grow_xallreduce", c_int, [c_vp, ctypes.POINTER(c_vp), c_ll, c_int, c_int, c_vp, c_vp, c_ll, c_int,
                                     ctypes.c_uint, c_vp]),
    ("yabt_grow_xerr", c_int, [c_vp, ctypes.POINTER(ctypes.c_uint)]),
    ("yabt_grower_set_feature_slice", c_int, [c_vp, c_int, c_int]),
    ("yabt_grow_scan", c_int, [c_vp, ctypes.POINTER(TreeArgs), c_int, c_vp]),
    ("yabt_grow_choose", c_int, [c_vp, ctypes.POINTER(TreeArgs), c_int, c_vp]),
    ("yabt_grow_xreduce_sliced", c_int, [c_vp, ctypes.POINTER(c_vp), c_int, c_int, c_int, ctypes.c_uint, c_vp]),
    ("yabt_grow_xgather", c_int, [c_vp, ctypes.POINTER(c_vp), c_int, c_int, c_int, ctypes.c_uint, c_ll, c_vp]),
    ("yabt_grow_xgather_bytes", c_ll, [c_vp]),
    ("yabt_grow_level_loop_sharded", c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_ll, ctypes.c_uint, c_vp, c_vp]),
    ("yabt_grow_small_count", c_ll, [c_vp, c_int]),
    ("yabt_grow_leaf_rows", c_int, [c_vp] + [ctypes.POINTER(c_vp)] * 6),
    ("yabt_transpose", c_int, [c_vp, c_ll, c_int, c_vp, c_vp]),
    ("yabt_transpose_block", c_int, [c_vp, c_ll, c_int, c_vp, c_ll, c_vp]),
    ("yabt_hist_build_workspace_bytes", c_ll, [c_ll, c_int, c_int]),
    ("yabt_hist_build", c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_ll, c_int, c_int, c_int, c_vp, c_vp, c_vp,
                                c_ll, c_vp]),
    ("yabt_bin_fit_workspace_bytes", c_ll, [c_ll, c_int, c_ll]),
    ("yabt_bin_fit", c_int, [c_vp, c_ll, c_int, c_vp, c_ll, c_int, c_vp, c_ll, c_vp, c_vp, c_vp, c_vp, c_vp]),
    ("yabt_bin_fit_static_capacity", c_ll, []),
    ("yabt_bin_fit_static", c_int, [c_vp, c_ll, c_int, c_vp, c_ll, c_int, c_vp, c_vp, c_vp, c_vp, c_vp]),
    ("yabt_bin_median_hist", c_int, [c_vp, c_ll, c_int, c_int, c_vp, c_ll, c_vp]),
    ("yabt_bin_median_pick", c_int, [c_ll, c_int, c_int, c_vp, c_ll, c_vp]),
    ("yabt_bin_median_final", c_int, [c_int, c_vp, c_ll, c_vp, c_vp]),
    ("yabt_bin_median_bufs", c_int, [c_int, c_vp, ctypes.POINTER(c_vp), ctypes.POINTER(c_ll), ctypes.POINTER(c_vp)]),
    ("yabt_bin_fit_edges", c_int, [c_vp, c_ll, c_int, c_int, c_vp, c_ll, c_vp, c_vp, c_vp, c_vp]),
    ("yabt_bin_transform", c_int, [c_vp, c_ll, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    ("yabt_leafnet_workspace_bytes", c_ll, [c_ll, c_int, c_int]),
    ("yabt_leafnet_fit", c_int, [ctypes.POINTER(LeafNetArgs), c_vp, c_ll, c_vp]),
    ("yabt_leafnet_stage", c_int, [ctypes.POINTER(LeafNetArgs), c_int, c_vp, c_ll, c_vp]),
    ("yabt_leafnet_bufs", c_int, [ctypes.POINTER(LeafNetArgs), c_vp, c_ll, ctypes.POINTER(c_vp), ctypes.POINTER(c_ll),
                                  ctypes.POINTER(c_vp), ctypes.POINTER(c_ll), ctypes.POINTER(c_vp),
                                  ctypes.POINTER(c_ll)]),
    ("yabt_update_margin", c_int, [ctypes.POINTER(UpdateArgs), c_vp]),
    ("yabt_grad_init", c_int, [c_vp, c_vp, c_ll, c_int, c_vp, c_vp, c_vp]),
    ("yabt_column_stats", c_int, [c_vp, c_ll, c_int, c_vp, c_vp, c_vp]),
    ("yabt_column_sums", c_int, [c_vp, c_ll, c_ll, c_int, c_int, c_vp, c_vp]),
    ("yabt_column_finish", c_int, [c_vp, c_ll, c_int, c_vp, c_vp, c_vp]),
    ("yabt_interaction_update", c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_vp]),
    ("yabt_interaction_normalize", c_int, [c_vp, c_int, c_vp, c_vp]),
    ("yabt_predict_forest", c_int, [c_vp, c_ll, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                    c_vp, c_int, c_vp, c_vp, c_vp, c_float, c_vp, c_vp]),
    ("yabt_apply_tree", c_int, [c_vp, c_ll, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    ("yabt_impute_rows", c_int, [c_vp, c_ll, c_int, c_vp, c_vp]),
]


class YabtError(RuntimeError):
    pass


def load():
    """Load the shared library (once). Raises if it is missing."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        if not os.path.exists(LIB_PATH):
            raise YabtError(f"{LIB_PATH} is missing: build it with `python -m yabt_b200.build` "
                            "(the CUDA path has no fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
        return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    load().yabt_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        raise YabtError(f"{what}: yabt error {rc}: {last_error()}")


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_ptr(stream=None) -> int | None:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream or None
