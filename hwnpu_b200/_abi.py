"""ctypes view of include/hwnpu_cuda.h and the loader of libhwnpu_cuda.so.

The loader follows the reference's purego binding of its native shims
(internal/backend/amdxrt/shim.go:81-150): a library path from the environment
(HWNPU_CUDA_SHIM, like HWNPU_XRTSHIM) or the in-tree build, an ABI check, and the
error protocol where a non-NULL char* is an error message the caller frees.
There is no fallback: without the library every call raises.
"""

import ctypes as C
import os

HC_ABI = 2

HC_STATE_COMPLETED, HC_STATE_ERROR, HC_STATE_TIMEOUT = 4, 5, 8
HC_INFO_NAME, HC_INFO_PCI_BUS_ID, HC_INFO_ARCH, HC_INFO_MEMORY, HC_INFO_SMS, HC_INFO_DRIVER = range(6)
HC_BUF_DEVICE, HC_BUF_HOST = 0, 1
HC_SYNC_TO_DEVICE, HC_SYNC_FROM_DEVICE = 0, 1
HC_FMT_NONE, HC_FMT_F16, HC_FMT_BF16 = -1, 0, 1
HC_FMT_INT8_ROW, HC_FMT_INT4_SYM_G32, HC_FMT_INT4_ASYM_G32, HC_FMT_MXFP4 = 2, 3, 4, 5
HC_ARCH_QWEN3, HC_ARCH_GPTOSS = 1, 2
HC_MODEL_QK_NORM, HC_MODEL_TIED, HC_MODEL_NORM_SCALE, HC_MODEL_ATTN_BIAS = 1, 2, 4, 8
HC_KV_F16, HC_KV_INT8_PAGED = 0, 1
HC_SESSION_NO_GRAPH = 1
HC_STEP_ALL_ROWS = 1

_p = C.c_void_p


class LinearDesc(C.Structure):
    _fields_ = [("format", C.c_int32), ("rows", C.c_uint32), ("cols", C.c_uint32),
                ("data", _p), ("scales", _p), ("zeros", _p), ("exps", _p), ("bias", _p)]


class LayerDesc(C.Structure):
    _fields_ = [("input_norm", _p), ("post_norm", _p), ("q_norm", _p), ("k_norm", _p),
                ("q", LinearDesc), ("k", LinearDesc), ("v", LinearDesc), ("o", LinearDesc),
                ("gate", LinearDesc), ("up", LinearDesc), ("down", LinearDesc),
                ("sinks", _p), ("sliding_window", C.c_uint32), ("pad_", C.c_uint32),
                ("router", LinearDesc), ("experts_gate_up", LinearDesc), ("experts_down", LinearDesc)]


class ModelDesc(C.Structure):
    _fields_ = [("abi", C.c_uint32), ("arch", C.c_uint32), ("flags", C.c_uint32),
                ("hidden", C.c_uint32), ("inter", C.c_uint32), ("layers", C.c_uint32),
                ("heads", C.c_uint32), ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("vocab", C.c_uint32), ("experts", C.c_uint32), ("top_k", C.c_uint32),
                ("norm_eps", C.c_double), ("rope_theta", C.c_double), ("yarn_factor", C.c_double),
                ("yarn_beta_fast", C.c_double), ("yarn_beta_slow", C.c_double),
                ("yarn_original", C.c_uint32), ("yarn_truncate", C.c_uint32),
                ("swiglu_alpha", C.c_double), ("swiglu_limit", C.c_double),
                ("embed", _p), ("final_norm", _p), ("head", LinearDesc), ("layer", C.POINTER(LayerDesc))]


class SessionOpts(C.Structure):
    _fields_ = [("max_context", C.c_uint32), ("max_seqs", C.c_uint32), ("max_step", C.c_uint32),
                ("kv_format", C.c_uint32), ("page_size", C.c_uint32), ("flags", C.c_uint32)]


class Stats(C.Structure):
    _fields_ = [("steps", C.c_uint64), ("tokens", C.c_uint64), ("launches", C.c_uint64),
                ("weight_bytes", C.c_uint64), ("kv_bytes", C.c_uint64), ("last_step_us", C.c_double)]


class HcError(RuntimeError):
    """An error string returned by the library."""


_u16p, _i32p, _f32p, _u8p = C.POINTER(C.c_uint16), C.POINTER(C.c_int32), C.POINTER(C.c_float), C.POINTER(C.c_uint8)
_err = C.c_void_p  # char*, freed by hc_free_error

# name: (restype, argtypes); every function declared in include/hwnpu_cuda.h
SIGNATURES = {
    "hc_abi": (C.c_int, []),
    "hc_free_error": (None, [C.c_void_p]),
    "hc_device_count": (_err, [C.POINTER(C.c_uint32)]),
    "hc_device_open": (_err, [C.c_uint32, C.POINTER(C.c_void_p)]),
    "hc_device_free": (None, [C.c_void_p]),
    "hc_device_info": (_err, [C.c_void_p, C.c_int, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "hc_buf_alloc": (_err, [C.c_void_p, C.c_uint64, C.c_int, C.POINTER(C.c_void_p)]),
    "hc_buf_free": (None, [C.c_void_p]),
    "hc_buf_map": (_err, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "hc_buf_address": (C.c_uint64, [C.c_void_p]),
    "hc_buf_sync": (_err, [C.c_void_p, C.c_int, C.c_uint64, C.c_uint64]),
    "hc_model_load": (_err, [C.c_void_p, C.POINTER(ModelDesc), C.POINTER(C.c_void_p)]),
    "hc_model_free": (None, [C.c_void_p]),
    "hc_model_weight_bytes": (C.c_uint64, [C.c_void_p]),
    "hc_session_new": (_err, [C.c_void_p, C.POINTER(SessionOpts), C.POINTER(C.c_void_p)]),
    "hc_session_free": (None, [C.c_void_p]),
    "hc_step": (_err, [C.c_void_p, _i32p, _i32p, _i32p, C.c_int32, C.c_int32, _u16p, _i32p,
                       C.c_uint32, _i32p]),
    "hc_speculate": (_err, [C.c_void_p, C.c_int32, _i32p, C.c_int32, _i32p, _i32p, _u16p,
                            C.c_uint32, _i32p]),
    "hc_generate": (_err, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, _i32p, C.c_uint32, _i32p]),
    "hc_session_stream": (_err, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "hc_seq_reset": (_err, [C.c_void_p, C.c_int32]),
    "hc_seq_truncate": (_err, [C.c_void_p, C.c_int32, C.c_int32]),
    "hc_seq_pos": (_err, [C.c_void_p, C.c_int32, _i32p]),
    "hc_seq_export_rows": (_err, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                  C.c_uint64, C.POINTER(C.c_uint64)]),
    "hc_seq_import_rows": (_err, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                  C.c_uint64]),
    "hc_stats_get": (_err, [C.c_void_p, C.POINTER(Stats)]),
    "hc_set_fault": (_err, [C.c_char_p]),
    "hc_synth_normal": (_err, [C.c_uint64, C.c_char_p, _f32p, _f32p, C.c_uint64]),
    "hc_synth_tokens": (_err, [C.c_uint64, C.c_int32, _i32p, C.c_uint64]),
    "hc_quantize_linear": (_err, [_f32p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_int32, C.c_int32,
                                  _u8p, _u16p]),
    "hc_quantize_int4_asym": (_err, [_f32p, C.c_uint32, C.c_uint32, _u8p, _u16p, _u16p]),
    "hc_mxfp4_encode": (_err, [_f32p, C.c_uint32, C.c_uint32, _u8p, _u8p]),
    "hc_f32_to_f16": (None, [_f32p, _u16p, C.c_uint64]),
    "hc_f16_to_f32": (None, [_u16p, _f32p, C.c_uint64]),
    "hc_linear_load": (_err, [C.c_void_p, C.POINTER(LinearDesc), C.POINTER(C.c_void_p)]),
    "hc_linear_free": (None, [C.c_void_p]),
    "hc_linear_dequant": (_err, [C.c_void_p, C.c_uint32, C.c_uint32, _f32p]),
    "hc_linear_run": (_err, [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p]),
    "hc_attention_run": (_err, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                C.c_int32, _f32p, C.c_void_p]),
    "hc_device_check": (_err, [C.c_void_p]),
    "hc_attention_run_static": (_err, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                       C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                       C.c_int32, _f32p, C.c_void_p]),
    "hc_argmax_run": (_err, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]),
    "hc_route_run": (_err, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p,
                            C.c_void_p]),
}

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libhwnpu_cuda.so")
_lib = None


def lib_path():
    return os.environ.get("HWNPU_CUDA_SHIM") or LIB_PATH


def lib():
    """The loaded library, bound and ABI-checked (amdxrt/shim.go:110-140). Raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.exists(path):
        raise HcError(f"libhwnpu_cuda.so not found at {path}: build it (python -c 'import __graft_entry__ as g; g.build()')")
    L = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    if L.hc_abi() != HC_ABI:
        raise HcError(f"{path}: ABI {L.hc_abi()}, this binding wants {HC_ABI}")
    _lib = L
    return L


def check(err):
    """The error protocol: NULL is success, else the message is raised and freed."""
    if err:
        msg = C.cast(err, C.c_char_p).value.decode(errors="replace")
        lib().hc_free_error(err)
        raise HcError(msg)
