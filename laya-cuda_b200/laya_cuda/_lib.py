"""ctypes binding of liblaya_b200.so, the sm_100a execution library (include/laya_b200.h).

The library is built in-tree next to this file (see build.py).  There is no fallback: if the
library is missing, importing the runtime raises, so a run never silently executes elsewhere.
"""
import ctypes as ct
from pathlib import Path

LIB_NAME = "liblaya_b200.so"
LIB_PATH = Path(__file__).with_name(LIB_NAME)

OK, ERR_INVALID, ERR_CUDA, ERR_DEVICE, ERR_STATE, ERR_NO_DEVICE = range(6)
DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
PRECISION_BF16, PRECISION_F16 = 0, 1

# Every symbol declared in include/laya_b200.h.
EXPORTS = (
    "laya_create", "laya_load_tensor", "laya_load_checkpoint", "laya_scan_checkpoint", "laya_finalize", "laya_predict", "laya_submit", "laya_collect",
    "laya_shape_class",
    "laya_forward_device", "laya_packed_ints", "laya_pack", "laya_reserve", "laya_stream", "laya_set_profiling",
    "laya_profile_read", "laya_read_tensor", "laya_cached_shapes", "laya_pool_bytes", "laya_destroy",
    "laya_last_error", "laya_set_launch_options", "laya_op_gemm", "laya_op_gemm_ln", "laya_interleave_geglu", "laya_op_attention", "laya_op_attention_gathered",
    "laya_attention_tiles", "laya_op_embed_norm", "laya_op_head_tail", "laya_op_norm", "laya_op_gemm_residual_static",
)
STATIC_SCRATCH_FLOATS = 4 * 1024 * 1024


class Config(ct.Structure):
    _fields_ = [("vocab", ct.c_int32), ("width", ct.c_int32), ("heads", ct.c_int32), ("layers", ct.c_int32),
                ("intermediate", ct.c_int32), ("global_every", ct.c_int32), ("window", ct.c_int32),
                ("theta_global", ct.c_float), ("theta_local", ct.c_float), ("eps", ct.c_float),
                ("max_len", ct.c_int32), ("head_layers", ct.c_int32), ("n_act", ct.c_int32),
                ("precision", ct.c_int32)]


class Metrics(ct.Structure):
    _fields_ = [("gpu_ms", ct.c_float), ("rows", ct.c_int32), ("batch", ct.c_int32), ("options", ct.c_int32),
                ("cache_miss", ct.c_int32), ("graph_capture", ct.c_int32), ("graph_replay", ct.c_int32),
                ("kernel_launches", ct.c_int32), ("owned_gpu_bytes", ct.c_uint64)]


_lib = None


def load():
    """Loads the library once and declares its signatures."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.is_file():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m laya_cuda.build` "
                           "(nvcc, sm_100a); there is no CPU fallback")
    lib = ct.CDLL(str(LIB_PATH))
    p, i, i32p, i64p, f32p = ct.c_void_p, ct.c_int, ct.POINTER(ct.c_int32), ct.POINTER(ct.c_int64), ct.POINTER(ct.c_float)
    sig = {
        "laya_create": (i, [ct.POINTER(Config), i, i, ct.POINTER(p)]),
        "laya_load_tensor": (i, [p, ct.c_char_p, i, i64p, i, p]),
        "laya_load_checkpoint": (i, [p, ct.c_char_p]),
        "laya_scan_checkpoint": (i, [ct.c_char_p, i64p, i64p]),
        "laya_finalize": (i, [p]),
        "laya_predict": (i, [p, p, p, p, p, p, i, i, p, p, ct.POINTER(Metrics)]),
        "laya_submit": (i, [p, p, p, p, p, p, i, i, i64p]),
        "laya_collect": (i, [p, ct.c_int64, p, p, ct.POINTER(Metrics)]),
        "laya_shape_class": (i, [p, p, i, i32p, i32p, i32p]),
        "laya_forward_device": (i, [p, p, i, i, i, i, p, p]),
        "laya_packed_ints": (ct.c_int64, [i, i, i]),
        "laya_pack": (i, [p, p, p, p, p, i, i, i, i, i, p]),
        "laya_reserve": (i, [p, i, i, i]),
        "laya_stream": (p, [p]),
        "laya_set_profiling": (i, [p, i]),
        "laya_profile_read": (i, [p, i, ct.POINTER(ct.c_double), i64p, ct.POINTER(ct.c_double)]),
        "laya_read_tensor": (i, [p, ct.c_char_p, f32p, ct.c_int64]),
        "laya_cached_shapes": (i, [p, i32p]),
        "laya_pool_bytes": (i, [p, ct.POINTER(ct.c_uint64), ct.POINTER(ct.c_uint64)]),
        "laya_destroy": (i, [p]),
        "laya_last_error": (ct.c_char_p, [p]),
        "laya_set_launch_options": (i, [i, ct.c_uint64]),
        "laya_op_gemm": (i, [i, i, p, p, i, i, i, p, i, p, i, p, i, p, i, p, i, i, p, p]),
        "laya_op_gemm_ln": (i, [i, p, p, i, i, i, p, i, p, p, p, ct.c_float, p, i, p, p]),
        "laya_interleave_geglu": (i, [p, p, i, i]),
        "laya_op_attention": (i, [i, i, p, p, p, i, p, p, i, i, i, p, p]),
        "laya_op_attention_gathered": (i, [i, p, p, p, i, p, p, i, i, i, p, p]),
        "laya_attention_tiles": (i, [p, p, i, i, i, p, i]),
        "laya_op_embed_norm": (i, [i, p, p, p, ct.c_float, i, i, i, p, p, p, p]),
        "laya_op_norm": (i, [i, p, p, i, p, p, ct.c_float, p, i, i, p]),
        "laya_op_head_tail": (i, [i, p, p, p, i, i, i, p, p, p, p, p, p, i, p, p, p, p, p, p]),
        "laya_op_gemm_residual_static": (i, [i, p, p, i, i, i, i, p, p, p, p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    _lib = lib
    return lib


def check(code, handle=None):
    """Maps a status code to the reference's exception types (ValueError / RuntimeError)."""
    if code == OK:
        return
    message = load().laya_last_error(handle).decode(errors="replace")
    if code == ERR_INVALID:
        raise ValueError(message)
    raise RuntimeError(message or f"laya_b200 error {code}")
