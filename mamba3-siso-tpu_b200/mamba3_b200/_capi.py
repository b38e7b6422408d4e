"""ctypes binding of ``include/m3_siso.h`` (libm3siso.so).

This is the whole host->device boundary: plain structs of pointers and sizes, one call
per kernel, an int status and a thread-local message.  The library is loaded from this
package's ``_lib/`` directory; there is no fallback -- if it is missing the import of any
op fails loudly.
"""

from __future__ import annotations

import ctypes
import os

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libm3siso.so")

M3_OK = 0
M3_ERR_ARG = -1
M3_ERR_SHAPE = -2
M3_ERR_UNSUPPORTED = -3
M3_ERR_WORKSPACE = -4
M3_ERR_LAUNCH = -5
M3_DTYPE_F32 = 0
M3_DTYPE_BF16 = 1
M3_POLICY_F32 = 0
M3_POLICY_BF16 = 1

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float


class M3Dims(ctypes.Structure):
    _fields_ = [("batch", _i32), ("seqlen", _i32), ("nheads", _i32), ("state_dim", _i32),
                ("headdim", _i32), ("n_angles", _i32), ("chunk", _i32)]


class M3Strides(ctypes.Structure):
    _fields_ = [("b", _i64), ("h", _i64), ("l", _i64)]


class M3FwdArgs(ctypes.Structure):
    _fields_ = [
        ("dims", M3Dims), ("io_dtype", _i32), ("policy", _i32), ("raw", _i32), ("a_floor", _f32),
        ("q", _vp), ("k", _vp), ("q_st", M3Strides), ("k_st", M3Strides),
        ("v", _vp), ("v_st", M3Strides), ("z", _vp), ("z_st", M3Strides),
        ("adt", _vp), ("gamma", _vp), ("scale", _vp), ("phi", _vp),
        ("dt_raw", _vp), ("a_raw", _vp), ("trap_raw", _vp), ("raw_st", M3Strides),
        ("angles", _vp), ("ang_st", M3Strides), ("dt_bias", _vp),
        ("q_bias", _vp), ("k_bias", _vp), ("d_skip", _vp),
        ("seed_ssm", _vp), ("seed_k", _vp), ("seed_v", _vp), ("seed_coef", _vp), ("seed_phi", _vp),
        ("y", _vp), ("y_st", M3Strides),
        ("final_ssm", _vp), ("final_k", _vp), ("final_v", _vp), ("final_phi", _vp),
        ("ybar", _vp), ("chunk_states", _vp), ("chunk_states_dtype", _i32),
        ("kernel", _i32), ("bwd_states", _vp), ("bwd_states_bytes", ctypes.c_size_t),
        ("fwd_workspace", _vp), ("fwd_workspace_bytes", ctypes.c_size_t),
        ("fwd_workspace_ready", ctypes.c_int32),
    ]


class M3SplitPrepArgs(ctypes.Structure):
    _fields_ = [("batch", _i32), ("seqlen", _i32), ("nheads", _i32), ("n_angles", _i32), ("segments", _i32),
                ("a_floor", _f32), ("dt_raw", _vp), ("a_raw", _vp), ("trap_raw", _vp), ("raw_st", M3Strides),
                ("angles", _vp), ("ang_st", M3Strides), ("dt_bias", _vp), ("partial", _vp), ("coef", _vp)]


class M3SplitCarryArgs(ctypes.Structure):
    _fields_ = [("batch", _i32), ("nheads", _i32), ("segments", _i32), ("tiles", _i32), ("state_dim", _i32),
                ("headdim", _i32), ("n_angles", _i32), ("partial", _vp), ("a_seg", _vp), ("coef", _vp), ("s_loc", _vp),
                ("k_last", _vp), ("v_last", _vp), ("seed_ssm", _vp), ("seed_k", _vp), ("seed_v", _vp), ("seed_phi", _vp),
                ("phi_in", _vp), ("c_ssm", _vp), ("c_k", _vp), ("c_v", _vp)]


M3_SPLIT_TILE = 64

M3_KERNEL_AUTO = 0
M3_KERNEL_GENERIC = 1
M3_KERNEL_TENSORCORE = 2
M3_KERNEL_TENSORCORE_V1 = 3


class M3BwdArgs(ctypes.Structure):
    _fields_ = [
        ("dims", M3Dims), ("io_dtype", _i32), ("policy", _i32), ("raw", _i32), ("a_floor", _f32),
        ("q", _vp), ("k", _vp), ("q_st", M3Strides), ("k_st", M3Strides),
        ("v", _vp), ("v_st", M3Strides), ("z", _vp), ("z_st", M3Strides),
        ("adt", _vp), ("gamma", _vp), ("scale", _vp), ("phi", _vp),
        ("dt_raw", _vp), ("a_raw", _vp), ("trap_raw", _vp), ("raw_st", M3Strides),
        ("angles", _vp), ("ang_st", M3Strides), ("dt_bias", _vp),
        ("q_bias", _vp), ("k_bias", _vp), ("d_skip", _vp),
        ("seed_ssm", _vp), ("seed_k", _vp), ("seed_v", _vp), ("seed_coef", _vp), ("seed_phi", _vp),
        ("dy", _vp), ("dy_st", M3Strides),
        ("dfinal_ssm", _vp), ("dfinal_k", _vp), ("dfinal_v", _vp), ("dfinal_phi", _vp),
        ("dq", _vp), ("dk", _vp), ("dv", _vp), ("dz", _vp),
        ("dadt", _vp), ("dgamma", _vp), ("dscale", _vp), ("dphi", _vp),
        ("ddt_raw", _vp), ("da_raw", _vp), ("dtrap_raw", _vp), ("dangles", _vp), ("ddt_bias", _vp),
        ("dq_bias", _vp), ("dk_bias", _vp), ("dd_skip", _vp),
        ("dseed_ssm", _vp), ("dseed_k", _vp), ("dseed_v", _vp), ("dseed_coef", _vp), ("dseed_phi", _vp),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
        ("kernel", _i32), ("grad_dtype", _i32), ("states_ready", _i32), ("dv_st", M3Strides), ("dz_st", M3Strides),
    ]


class M3DecodeArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i32), ("nheads", _i32), ("state_dim", _i32), ("headdim", _i32), ("n_angles", _i32),
        ("io_dtype", _i32), ("policy", _i32), ("raw", _i32), ("a_floor", _f32),
        ("q", _vp), ("k", _vp), ("qk_stride_b", _i64),
        ("v", _vp), ("z", _vp), ("vz_stride_b", _i64),
        ("adt", _vp), ("dt", _vp), ("lam", _vp),
        ("dt_raw", _vp), ("a_raw", _vp), ("trap_raw", _vp), ("raw_stride_b", _i64),
        ("dt_bias", _vp), ("angles", _vp), ("ang_stride_b", _i64),
        ("q_bias", _vp), ("k_bias", _vp), ("d_skip", _vp),
        ("ssm", _vp), ("state_k", _vp), ("state_v", _vp), ("phi", _vp),
        ("y", _vp),
        ("scalar_dtype", _i32), ("q_norm_w", _vp), ("k_norm_w", _vp), ("norm_eps", _f32),
    ]


class M3SampleArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i32), ("vocab", _i32), ("logits_dtype", _i32), ("logits_ld", _i64), ("logits", _vp),
        ("temperature", _f32), ("top_p", _f32), ("rep_penalty", _f32), ("seed", ctypes.c_uint64),
        ("counter", _vp), ("seen_count", _vp), ("window", _vp), ("window_state", _vp), ("rep_window", _i32),
        ("stop_ids", _vp), ("n_stop", _i32), ("done", _vp), ("out_token", _vp), ("history", _vp),
        ("history_cap", _i64), ("scratch", _vp), ("probs_out", _vp), ("probs_ld", _i64),
    ]


class M3GemvArgs(ctypes.Structure):
    _fields_ = [
        ("m", _i32), ("k", _i32), ("n", _i32), ("x_mode", _i32), ("x", _vp), ("x_ld", _i64),
        ("norm_w", _vp), ("eps", _f32), ("w", _vp), ("w_ld", _i64), ("residual", _vp), ("r_ld", _i64),
        ("out", _vp), ("out_ld", _i64), ("scratch", _vp), ("tickets", _vp),
    ]


class M3GemmArgs(ctypes.Structure):
    _fields_ = [
        ("m", _i32), ("n", _i32), ("k", _i32), ("w_kmajor", _i32), ("ksplit", _i32), ("reserved", _i32),
        ("a", _vp), ("lda", _i64), ("w", _vp),
        ("ldw", _i64), ("residual", _vp), ("ldr", _i64), ("out", _vp), ("ldo", _i64),
    ]


EXPORTS = ("m3_siso_fwd", "m3_siso_fwd_workspace_size", "m3_siso_bwd", "m3_siso_bwd_workspace_size", "m3_siso_decode",
           "m3_last_error", "m3_version", "m3_siso_bwd_noalloc", "m3_siso_bwd_noalloc_scratch_bytes",
           "m3_device_error", "m3_copy2d_async", "m3_rms_norm", "m3_rms_norm_bwd", "m3_sample_tokens", "m3_gemv_bf16",
           "m3_gemv_scratch_floats", "m3_siso_fwd_saves_states", "m3_gated_act_bf16", "m3_siso_split_prep",
           "m3_siso_split_carry", "m3_gemm_bf16")

_lib = None


def lib():
    """Load libm3siso.so once; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise RuntimeError(
                f"libm3siso.so not found at {_LIB_PATH}; build it with "
                "`python mamba3-siso-tpu_b200/build.py` (there is no fallback path)")
        L = ctypes.CDLL(_LIB_PATH)
        L.m3_siso_fwd.argtypes = [ctypes.POINTER(M3FwdArgs), _vp]
        L.m3_siso_fwd.restype = ctypes.c_int
        L.m3_siso_fwd_saves_states.argtypes = [ctypes.POINTER(M3FwdArgs)]
        L.m3_siso_fwd_saves_states.restype = ctypes.c_int
        L.m3_siso_bwd.argtypes = [ctypes.POINTER(M3BwdArgs), _vp]
        L.m3_siso_bwd.restype = ctypes.c_int
        L.m3_siso_split_prep.argtypes = [ctypes.POINTER(M3SplitPrepArgs), _vp]
        L.m3_siso_split_prep.restype = ctypes.c_int
        L.m3_siso_split_carry.argtypes = [ctypes.POINTER(M3SplitCarryArgs), _vp]
        L.m3_siso_split_carry.restype = ctypes.c_int
        L.m3_siso_fwd_workspace_size.argtypes = [ctypes.POINTER(M3Dims)]
        L.m3_siso_fwd_workspace_size.restype = ctypes.c_size_t
        L.m3_siso_bwd_workspace_size.argtypes = [ctypes.POINTER(M3Dims)]
        L.m3_siso_bwd_workspace_size.restype = ctypes.c_size_t
        L.m3_siso_decode.argtypes = [ctypes.POINTER(M3DecodeArgs), _vp]
        L.m3_siso_decode.restype = ctypes.c_int
        L.m3_last_error.argtypes = []
        L.m3_last_error.restype = ctypes.c_char_p
        L.m3_version.argtypes = []
        L.m3_version.restype = ctypes.c_int
        L.m3_device_error.argtypes = [ctypes.c_int]
        L.m3_device_error.restype = ctypes.c_int
        L.m3_sample_tokens.argtypes = [ctypes.POINTER(M3SampleArgs), _vp]
        L.m3_sample_tokens.restype = ctypes.c_int
        L.m3_gated_act_bf16.argtypes = [_vp, ctypes.c_int64, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, _vp]
        L.m3_gated_act_bf16.restype = ctypes.c_int
        L.m3_gemv_bf16.argtypes = [ctypes.POINTER(M3GemvArgs), _vp]
        L.m3_gemv_bf16.restype = ctypes.c_int
        L.m3_gemm_bf16.argtypes = [ctypes.POINTER(M3GemmArgs), _vp]
        L.m3_gemm_bf16.restype = ctypes.c_int
        L.m3_gemv_scratch_floats.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]
        L.m3_gemv_scratch_floats.restype = ctypes.c_size_t
        L.m3_copy2d_async.argtypes = [_vp, ctypes.c_size_t, _vp, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t, _vp]
        L.m3_copy2d_async.restype = ctypes.c_int
        L.m3_rms_norm.argtypes = [_vp, ctypes.c_int64, _vp, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                  ctypes.c_float, ctypes.c_int32, ctypes.c_int32, _vp, _vp]
        L.m3_rms_norm.restype = ctypes.c_int
        L.m3_rms_norm_bwd.argtypes = [_vp, ctypes.c_int64, _vp, _vp, _vp, ctypes.c_int64, _vp, ctypes.c_int64, _vp,
                                      ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _vp]
        L.m3_rms_norm_bwd.restype = ctypes.c_int
        _lib = L
    return _lib


def library_path() -> str:
    return _LIB_PATH


class M3Error(ValueError):
    """A non-zero status from the library (subclasses ValueError like the reference's
    argument errors)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def check(rc: int):
    if rc != M3_OK:
        raise M3Error(rc, lib().m3_last_error().decode())
