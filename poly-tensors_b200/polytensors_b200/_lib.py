"""ctypes binding of libpolykern.so (the C ABI declared in include/polykern.h).

The library is loaded lazily on first use.  There is no fallback: if the shared
library is missing or CUDA is unavailable, every kernel entry point raises.
"""

import ctypes
import pathlib
import threading

LIB_PATH = pathlib.Path(__file__).resolve().parent / "lib" / "libpolykern.so"

# enum pk_dtype
PK_F32, PK_F64, PK_BF16, PK_F16, PK_C128 = 0, 1, 2, 3, 4
# enum pk_series_op
OP = dict(copy=0, affine=1, exp=2, log=3, sqrt=4, rsqrt=5, reciprocal=6, tanh=7, sigmoid=8, gelu=9, powi=10,
          add=32, mul=33, div=34, gelu_bwd=35, tanh_bwd=36, sigmoid_bwd=37)
PK_MAX_PLANES = 16

_i32, _i64, _sz, _vp = ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p
_pp = ctypes.POINTER(ctypes.c_void_p)
_p64 = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); every symbol declared in include/polykern.h
SIGNATURES = {
    "pk_version": (ctypes.c_char_p, []),
    "pk_last_error": (ctypes.c_char_p, []),
    "pk_device_status": (_i32, [_i32]),
    "pk_profile_enable": (_i32, [_i32]),
    "pk_launch_count": (_i64, [_i32]),
    "pk_profile_query": (_i32, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64)]),
    "pk_poly_gemm_workspace_size": (_sz, [_i32, _i32, _i64, _i64, _i64, _i64, _i32, _i32]),
    "pk_poly_gemm_workspace_query": (_i32, [_i32, _i32, _i64, _i64, _i64, _i64,
                                            _pp, _i64, _i64, _i64,
                                            _pp, _i64, _i64, _i64,
                                            _i32, _i32, ctypes.POINTER(ctypes.c_size_t)]),
    "pk_poly_gemm": (_i32, [_i32, _i32, _i64, _i64, _i64, _i64,
                            _pp, _i64, _i64, _i64,
                            _pp, _i64, _i64, _i64,
                            _pp, _i64, _i64,
                            _i32, _i32, _vp, _sz, _vp]),
    "pk_poly_gemm_banded": (_i32, [_i32, _i32, _i64, _i64, _i64, _i64,
                                   _pp, _i64, _i64, _i64,
                                   _pp, _i64, _i64, _i64,
                                   _pp, _i64, _i64,
                                   _i32, _i32, _i32, _i32, _i64, _vp, _sz, _vp]),
    "pk_poly_gemm_accumulate": (_i32, [_i32, _i32, _i64, _i64, _i64, _i64,
                                       _pp, _i64, _i64, _i64,
                                       _pp, _i64, _i64, _i64,
                                       _pp, _i64, _i64,
                                       _i32, _i32, _vp, _sz, _vp]),
    "pk_poly_gemm_hilo_workspace_query": (_i32, [_i32, _i64, _i64, _i64, _i64, _pp, _i64, _i64, _i64, _i32,
                                                 _pp, _i64, _i64, _i64, _i32, ctypes.POINTER(ctypes.c_size_t)]),
    "pk_poly_gemm_hilo": (_i32, [_i32, _i64, _i64, _i64, _i64, _pp, _i64, _i64, _i64, _i32,
                                 _pp, _i64, _i64, _i64, _i32, _pp, _i64, _i64, _i32, _i32, _i64, _vp, _sz, _vp]),
    "pk_series_map": (_i32, [_i32, _i32, _i32, _i32, _p64, _pp, _p64, _pp, _i32, _p64, _pp, _i32, _p64,
                             ctypes.c_double, ctypes.c_double, _vp]),
    "pk_series_map_complex": (_i32, [_i32, _i32, _i32, _i32, _p64, _pp, _p64, ctypes.c_uint32, _pp, _i32, _p64,
                                     ctypes.c_uint32, _pp, _i32, _p64, ctypes.c_uint32, ctypes.c_double,
                                     ctypes.c_double, _vp]),
    "pk_series_reduce": (_i32, [_i32, _i32, _i64, _i64, _i64, _pp, _pp, ctypes.c_double, _vp]),
    "pk_series_gather_rows": (_i32, [_i32, _i32, _i64, _i64, _vp, _pp, _i64, _i64, _pp, _vp]),
    "pk_series_scatter_add_rows": (_i32, [_i32, _i32, _i64, _i64, _vp, _i64, _pp, _i64, _i64, _pp, _vp]),
    "pk_rmsnorm_fwd": (_i32, [_i32, _i32, _i64, _i64, _pp, _i64, _pp, _i32, ctypes.c_double, _pp, _i64, _vp, _vp]),
    "pk_rmsnorm_bwd_workspace_size": (_sz, [_i32, _i32, _i64, _i64]),
    "pk_rmsnorm_bwd": (_i32, [_i32, _i32, _i64, _i64, _pp, _i64, _pp, _i32, _pp, _i64, _vp, _pp, _i64, _pp,
                              _vp, _sz, _vp]),
    "pk_softmax_fwd": (_i32, [_i32, _i32, _i64, _i64, _pp, _i64, _i32, _pp, _i64, _vp]),
    "pk_softmax_bwd": (_i32, [_i32, _i32, _i64, _i64, _pp, _i64, _pp, _i64, _i32, _pp, _i64, _vp]),
    "pk_cross_entropy_fwd": (_i32, [_i32, _i32, _i64, _i64, _pp, _i64, _vp, _i64, ctypes.c_double, _pp, _vp,
                                    _vp]),
    "pk_cross_entropy_bwd": (_i32, [_i32, _i32, _i64, _i64, _pp, _i64, _vp, _i64, ctypes.c_double, _vp, _pp,
                                    _pp, _i64, _vp]),
    "pk_attn_probs": (_i32, [_i32, _i32, _i64, _i64, _i64, _pp, _i64, ctypes.c_double, _i32, _i64, _pp, _i64,
                             _vp, _vp]),
    "pk_attn_dscores": (_i32, [_i32, _i32, _i64, _i64, _pp, _i64, _pp, _i64, _vp, ctypes.c_double, _pp, _i64,
                               _vp]),
    "pk_scaled_from": (_i32, [_i32, _i32, _i64, _pp, _pp, _pp, ctypes.c_int32, _vp]),
    "pk_scaled_to": (_i32, [_i32, _i32, _i32, _i64, _pp, _pp, ctypes.c_int32, _pp, _vp]),
    "pk_scaled_series_map": (_i32, [_i32, _i32, _i32, _i32, _p64, _pp, _pp, _p64, _pp, _pp, _i32, _p64,
                                    _pp, _pp, _i32, _p64, ctypes.c_double, ctypes.c_double, _vp]),
    "pk_scaled_reduce": (_i32, [_i32, _i32, _i64, _i64, _i64, _pp, _pp, _pp, _pp, _vp]),
    "pk_attn_dsum": (_i32, [_i32, _i32, _i64, _i64, _pp, _i64, _pp, _i64, _vp, _vp]),
    "pk_split_hilo": (_i32, [_i32, _i64, _pp, _pp, _vp]),
    "pk_attn_probs_hilo": (_i32, [_i32, _i64, _i64, _i64, _pp, _i64, ctypes.c_double, _i32, _i64, _pp, _i64,
                                  _vp, _vp]),
    "pk_attn_dscores_hilo": (_i32, [_i32, _i64, _i64, _pp, _i64, _pp, _i64, _vp, ctypes.c_double, _pp, _i64,
                                    _vp]),
    "pk_flash_attn_fwd": (_i32, [_i32, _i32, _i64, _i64, _i64, _i64, _pp, _pp, _pp, _pp, _i32, ctypes.c_double,
                                 _vp, _vp]),
    "pk_attn_probs_gemm": (_i32, [_i32, _i32, _i64, _i64, _i64, _i64, _pp, _i64, _i64, _i64,
                                  _pp, _i64, _i64, _i64, _pp, _i64, _i64,
                                  _vp, _i64, ctypes.c_double, _i32, _i64, _vp]),
    "pk_attn_dscores_gemm": (_i32, [_i32, _i32, _i64, _i64, _i64, _i64, _pp, _i64, _i64, _i64,
                                    _pp, _i64, _i64, _i64, _pp, _i64, _i64,
                                    _vp, _i64, ctypes.c_double, _i32, _i64, _pp, _i64, _i64, _vp]),
    "pk_poly_gemm_noalloc": (_i32, [_i32, _i32, _i64, _i64, _i64, _i64,
                                    _pp, _i64, _i64, _i64,
                                    _pp, _i64, _i64, _i64,
                                    _pp, _i64, _i64,
                                    _i32, _i32, _vp]),
}

_lock = threading.Lock()
_lib = None


def load():
    """Load libpolykern.so and bind every exported entry point (raises if unavailable)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH} is not built; run polytensors_b200._build.build() "
                                   "(this package has no CPU fallback)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def last_error():
    return load().pk_last_error().decode(errors="replace")


def check(status, what):
    """Raise RuntimeError carrying pk_last_error() for a nonzero status."""
    if status != 0:
        raise RuntimeError(f"{what} failed ({status}): {last_error()}")


# Host-side companion of the launch timing: while it is on, the tensor-level wrappers add the
# algorithmic flops of every polynomial product they launch (benchmark rooflines).
_profile = {"on": False, "gemm_flops": 0.0}


def profile_enable(on=True):
    load().pk_profile_enable(1 if on else 0)
    _profile["on"] = bool(on)


def profiling():
    return _profile["on"]


def add_gemm_flops(flops):
    _profile["gemm_flops"] += flops


def take_gemm_flops():
    """Algorithmic flops of the polynomial products launched while timing was on, since the last call."""
    value, _profile["gemm_flops"] = _profile["gemm_flops"], 0.0
    return value


def profile_query(kernel):
    """(total milliseconds, launches) of the event-timed launches of ``kernel`` since the last query."""
    ms, n = ctypes.c_double(), ctypes.c_int64()
    check(load().pk_profile_query(kernel.encode(), ctypes.byref(ms), ctypes.byref(n)), "pk_profile_query")
    return ms.value, n.value


def launch_count(reset=False):
    """Kernels launched by the library so far (pk_launch_count); ``reset`` zeroes the count."""
    return load().pk_launch_count(1 if reset else 0)


def pointer_array(tensors):
    arr = (ctypes.c_void_p * len(tensors))(*[t.data_ptr() if t is not None else None for t in tensors])
    return ctypes.cast(arr, _pp), arr


def int64_array(values):
    arr = (ctypes.c_int64 * max(len(values), 1))(*values)
    return ctypes.cast(arr, _p64), arr
