"""ctypes binding of libsta.so (the C ABI declared in include/sta.h).

The library is loaded from ``sta/_lib/libsta.so`` inside this package.  There is no CPU
fallback: when the library is missing the import of any op raises immediately.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libsta.so")

STA_OK = 0
STA_DTYPE_F32 = 0
STA_DTYPE_BF16 = 1
SCORE = {"freq": 0, "margin": 1, "expmass": 2}
ADV = {"max": 0, "full": 1}

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_f32 = ctypes.c_float
c_vp = ctypes.c_void_p


class SelectArgs(ctypes.Structure):
    _fields_ = [("q_hi", c_vp), ("q_lo", c_vp), ("k_hi", c_vp), ("k_lo", c_vp),
                ("batch", c_i64), ("n_heads", c_i64), ("n_kv_heads", c_i64), ("n", c_i64),
                ("d", c_i32), ("tile", c_i32), ("sm_scale", c_f32), ("wmode", c_i32),
                ("tau", c_vp), ("max_only", c_i32), ("votes", c_vp), ("wvotes", c_vp),
                ("bits", c_vp), ("row_max", c_vp), ("row_count", c_vp),
                ("dca_chunk_len", c_i32), ("q_pos_base", c_i64),
                ("block_max", c_vp), ("block_max_bn", c_i32), ("wait_limit_ns", ctypes.c_uint64),
                ("screen_ws", c_vp), ("vote_hist", c_vp)]


class BuildArgs(ctypes.Structure):
    _fields_ = [("votes", c_vp), ("wvotes", c_vp), ("heads", c_i64), ("n", c_i64),
                ("tile", c_i32), ("k_max", c_i32), ("n_global", c_i32), ("n_local", c_i32),
                ("pct", c_f32), ("pos_scale", c_f32), ("select_score", c_i32),
                ("measure", c_i32), ("idx", c_vp), ("newpos_k", c_vp), ("newpos_q", c_vp),
                ("shared_size", c_vp), ("kept_size", c_vp), ("chosen", c_vp),
                ("overflow", c_vp), ("kpct_meas", c_vp), ("overflow20", c_vp),
                ("q_pos_base", c_i64), ("vote_hist", c_vp)]


class BuildPQArgs(ctypes.Structure):
    _fields_ = [("votes", c_vp), ("wvotes", c_vp), ("bits", c_vp), ("heads", c_i64),
                ("n", c_i64), ("tile", c_i32), ("k_max", c_i32), ("n_global", c_i32),
                ("n_local", c_i32), ("select_score", c_i32), ("idx", c_vp),
                ("newpos_k", c_vp), ("newpos_q", c_vp), ("mask", c_vp), ("usize", c_vp),
                ("kept_size", c_vp), ("overflow", c_vp), ("q_pos_base", c_i64)]


class BuildChunkArgs(ctypes.Structure):
    _fields_ = [("votes", c_vp), ("wvotes", c_vp), ("heads", c_i64), ("n", c_i64),
                ("tile", c_i32), ("k_max", c_i32), ("n_global", c_i32), ("n_local", c_i32),
                ("chunk_size", c_i32), ("n_chunk", c_i32), ("select_score", c_i32),
                ("chunk_agg", c_i32), ("idx", c_vp), ("newpos_k", c_vp), ("newpos_q", c_vp),
                ("mask", c_vp), ("usize", c_vp), ("kept_size", c_vp), ("q_pos_base", c_i64)]


class AttendArgs(ctypes.Structure):
    _fields_ = [("q", c_vp), ("q_stride_h", c_i64), ("q_stride_n", c_i64),
                ("k", c_vp), ("k_stride_h", c_i64), ("k_stride_n", c_i64),
                ("v", c_vp), ("v_stride_h", c_i64), ("v_stride_n", c_i64),
                ("out", c_vp), ("dtype", c_i32), ("batch", c_i64), ("n_heads", c_i64),
                ("n_kv_heads", c_i64), ("n", c_i64), ("d", c_i32), ("tile", c_i32),
                ("k_max", c_i32), ("idx", c_vp), ("newpos_k", c_vp), ("newpos_q", c_vp),
                ("mask", c_vp), ("kept_size", c_vp), ("inv_freq", c_vp),
                ("rope_scale", c_f32), ("sm_scale", c_f32), ("q_hi", c_vp), ("q_lo", c_vp),
                ("k_hi", c_vp), ("k_lo", c_vp), ("pos_scale_sel", c_f32),
                ("same_geometry", c_i32), ("rope_table", c_vp), ("rope_table_R", c_f32),
                ("rope_table_len", c_i64), ("q_pos_base", c_i64)]


class PQStreamArgs(ctypes.Structure):
    _fields_ = [("q", c_vp), ("q_stride_h", c_i64), ("q_stride_n", c_i64),
                ("k", c_vp), ("k_stride_h", c_i64), ("k_stride_n", c_i64),
                ("v", c_vp), ("v_stride_h", c_i64), ("v_stride_n", c_i64),
                ("out", c_vp), ("dtype", c_i32), ("batch", c_i64), ("n_heads", c_i64),
                ("n_kv_heads", c_i64), ("n", c_i64), ("d", c_i32), ("tile", c_i32),
                ("block_n", c_i32), ("bits", c_vp), ("block_max", c_vp), ("row_count", c_vp),
                ("n_global", c_i32), ("n_local", c_i32), ("inv_freq_c", c_vp),
                ("sm_scale", c_f32), ("pos_advance", c_i32), ("use_skip", c_i32),
                ("rope_table", c_vp), ("rope_table_R", c_f32), ("rope_table_len", c_i64),
                ("span", c_vp), ("kept", c_vp), ("blocks", c_vp), ("skipped", c_vp),
                ("q_pos_base", c_i64)]


class ForwardArgs(ctypes.Structure):
    _fields_ = [("q", c_vp), ("q_stride_h", c_i64), ("q_stride_n", c_i64),
                ("k", c_vp), ("k_stride_h", c_i64), ("k_stride_n", c_i64),
                ("v", c_vp), ("v_stride_h", c_i64), ("v_stride_n", c_i64),
                ("out", c_vp), ("dtype", c_i32), ("batch", c_i64), ("n_heads", c_i64),
                ("n_kv_heads", c_i64), ("n", c_i64), ("d", c_i32), ("tau", c_vp),
                ("inv_freq_a", c_vp), ("pos_scale_a", c_f32), ("rope_scale_a", c_f32),
                ("inv_freq_c", c_vp), ("pos_scale_c", c_f32), ("rope_scale_c", c_f32),
                ("sm_scale", c_f32), ("pct", c_f32), ("n_global", c_i32), ("n_local", c_i32),
                ("tile", c_i32), ("k_max", c_i32), ("select_score", c_i32),
                ("measure", c_i32), ("block_n", c_i32), ("pos_advance", c_i32),
                ("use_skip", c_i32), ("shared_size", c_vp), ("kept_size", c_vp),
                ("chosen", c_vp), ("overflow", c_vp), ("kpct_meas", c_vp),
                ("overflow20", c_vp), ("span", c_vp), ("kept_rows", c_vp), ("blocks", c_vp),
                ("skipped", c_vp), ("idx_out", c_vp), ("newpos_k_out", c_vp),
                ("newpos_q_out", c_vp), ("mask_out", c_vp), ("max_workspace_bytes", c_i64),
                ("stage_events", c_vp), ("same_geometry", c_i32), ("chunk_size", c_i32),
                ("n_chunk", c_i32), ("chunk_agg", c_i32), ("dca_chunk_size", c_i32),
                ("dca_local_window", c_i32), ("q_pos_base", c_i64)]


class DecodeArgs(ctypes.Structure):
    _fields_ = [("q", c_vp), ("q_stride_h", c_i64),
                ("k", c_vp), ("k_stride_h", c_i64), ("k_stride_n", c_i64),
                ("v", c_vp), ("v_stride_h", c_i64), ("v_stride_n", c_i64),
                ("out", c_vp), ("dtype", c_i32), ("batch", c_i64), ("n_heads", c_i64),
                ("n_kv_heads", c_i64), ("m", c_i64), ("d", c_i32), ("tau", c_vp),
                ("inv_freq_a", c_vp), ("pos_scale_a", c_f32), ("rope_scale_a", c_f32),
                ("inv_freq_c", c_vp), ("pos_scale_c", c_f32), ("rope_scale_c", c_f32),
                ("sm_scale", c_f32), ("mode", c_i32), ("n_global", c_i32), ("n_local", c_i32),
                ("k_max", c_i32), ("pct_decode", c_f32), ("block_n", c_i32),
                ("rope_table_a", c_vp), ("rope_table_a_R", c_f32), ("rope_table_a_len", c_i64),
                ("rope_table_c", c_vp), ("rope_table_c_R", c_f32), ("rope_table_c_len", c_i64),
                ("idx_out", c_vp), ("newpos_k_out", c_vp), ("newpos_q_out", c_vp),
                ("kept_out", c_vp), ("usize_out", c_vp), ("chunk_size", c_i32),
                ("n_chunk", c_i32), ("chunk_agg", c_i32), ("select_score", c_i32)]


DECODE = {"pi": 0, "rank": 1, "stream": 2, "chunk": 3}


class DcaArgs(ctypes.Structure):
    _fields_ = [("q", c_vp), ("q_stride_h", c_i64), ("q_stride_n", c_i64),
                ("k", c_vp), ("k_stride_h", c_i64), ("k_stride_n", c_i64),
                ("v", c_vp), ("v_stride_h", c_i64), ("v_stride_n", c_i64),
                ("out", c_vp), ("dtype", c_i32), ("batch", c_i64), ("n_heads", c_i64),
                ("n_kv_heads", c_i64), ("n", c_i64), ("d", c_i32), ("inv_freq", c_vp),
                ("rope_scale", c_f32), ("sm_scale", c_f32), ("chunk_size", c_i32),
                ("local_window", c_i32), ("q_pos_base", c_i64)]


# every symbol include/sta.h declares (checked by the CPU test suite)
EXPORTED = ["sta_last_error", "sta_version", "sta_tri_head_stride", "sta_rope_split",
            "sta_select", "sta_build_sets", "sta_build_sets_pq", "sta_gather_attend",
            "sta_pqstream_attend", "sta_shared_workspace_bytes", "sta_shared_forward",
            "sta_pq_union_workspace_bytes", "sta_pq_union_forward",
            "sta_pq_stream_workspace_bytes", "sta_pq_stream_forward", "sta_device_error",
            "sta_shared_forward_static", "sta_build_sets_chunk", "sta_chunk_workspace_bytes",
            "sta_chunk_forward", "sta_rope_split_dca", "sta_rope_table", "sta_tri_head_stride_q",
            "sta_decode_workspace_bytes", "sta_decode_forward", "sta_dca_workspace_bytes",
            "sta_dca_forward", "sta_select_screen_bytes"]

_lib = None


def lib():
    """Load libsta.so (once).  Raises RuntimeError when it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"libsta.so not built ({LIB_PATH}); run "
                           "`python sparse-thresholded-attention_b200/build.py`")
    L = ctypes.CDLL(LIB_PATH)
    L.sta_last_error.restype = ctypes.c_char_p
    L.sta_version.restype = ctypes.c_int
    L.sta_tri_head_stride.restype = c_i64
    L.sta_tri_head_stride.argtypes = [c_i64, c_i32]
    L.sta_tri_head_stride_q.restype = c_i64
    L.sta_tri_head_stride_q.argtypes = [c_i64, c_i32, c_i64]
    L.sta_rope_split.restype = ctypes.c_int
    L.sta_rope_split.argtypes = [c_vp, c_i32, c_i64, c_i64, c_i32, c_i64, c_i64, c_vp, c_f32,
                                 c_f32, c_vp, c_vp, c_vp]
    for name, st in (("sta_select", SelectArgs), ("sta_build_sets", BuildArgs),
                     ("sta_build_sets_pq", BuildPQArgs), ("sta_gather_attend", AttendArgs),
                     ("sta_build_sets_chunk", BuildChunkArgs),
                     ("sta_pqstream_attend", PQStreamArgs)):
        f = getattr(L, name)
        f.restype = ctypes.c_int
        f.argtypes = [ctypes.POINTER(st), c_vp]
    for v in ("shared", "pq_union", "pq_stream", "chunk"):
        f = getattr(L, f"sta_{v}_workspace_bytes")
        f.restype = ctypes.c_size_t
        f.argtypes = [ctypes.POINTER(ForwardArgs)]
        f = getattr(L, f"sta_{v}_forward")
        f.restype = ctypes.c_int
        f.argtypes = [ctypes.POINTER(ForwardArgs), c_vp, ctypes.c_size_t, c_vp]
    L.sta_rope_split_dca.restype = ctypes.c_int
    L.sta_rope_split_dca.argtypes = [c_vp, c_i32, c_i64, c_i64, c_i32, c_i64, c_i64, c_vp, c_f32,
                                     c_i32, c_i32, c_i32, c_vp, c_vp, c_vp]
    L.sta_rope_table.restype = ctypes.c_int
    L.sta_rope_table.argtypes = [c_vp, c_i32, c_f32, c_f32, c_i64, c_vp, c_vp]
    L.sta_decode_workspace_bytes.restype = ctypes.c_size_t
    L.sta_decode_workspace_bytes.argtypes = [ctypes.POINTER(DecodeArgs)]
    L.sta_decode_forward.restype = ctypes.c_int
    L.sta_decode_forward.argtypes = [ctypes.POINTER(DecodeArgs), c_vp, ctypes.c_size_t, c_vp]
    L.sta_dca_workspace_bytes.restype = ctypes.c_size_t
    L.sta_dca_workspace_bytes.argtypes = [ctypes.POINTER(DcaArgs)]
    L.sta_dca_forward.restype = ctypes.c_int
    L.sta_dca_forward.argtypes = [ctypes.POINTER(DcaArgs), c_vp, ctypes.c_size_t, c_vp]
    L.sta_select_screen_bytes.restype = ctypes.c_size_t
    L.sta_select_screen_bytes.argtypes = [ctypes.POINTER(SelectArgs)]
    L.sta_shared_forward_static.restype = ctypes.c_int
    L.sta_shared_forward_static.argtypes = [ctypes.POINTER(ForwardArgs), c_vp]
    L.sta_device_error.restype = ctypes.c_int
    L.sta_device_error.argtypes = [c_vp, ctypes.POINTER(c_i32)]
    _lib = L
    return L


class StaError(RuntimeError):
    pass


def check(rc: int, what: str):
    if rc != STA_OK:
        msg = lib().sta_last_error().decode(errors="replace")
        if rc in (1,):
            raise ValueError(f"{what}: {msg}")
        raise StaError(f"{what} failed (status {rc}): {msg}")
