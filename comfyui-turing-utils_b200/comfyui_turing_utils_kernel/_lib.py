"""ctypes binding of libctu_b200.so (the C ABI declared in include/ctu_b200.h).

The library is built in-tree (comfyui-turing-utils_b200/build.py).  There is no CPU
or eager fallback: if the library is missing or cannot be loaded, every operation
raises instead of computing anything.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libctu_b200.so"
_lock = threading.Lock()
_lib = None

CTU_OK = 0
CTU_ERR_INVALID_ARGUMENT = 1
CTU_ERR_UNSUPPORTED = 2
CTU_ERR_CUDA = 3

ACT_NONE = 0
ACT_SWIGLU = 1
ACT_GELU_TANH = 2

# name -> (restype, argtypes)
_vp, _i64, _i32, _u64, _f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_uint64, ctypes.c_float
SIGNATURES = {
    "ctu_version": (_i32, []),
    "ctu_last_error": (ctypes.c_char_p, []),
    "ctu_get_device_error": (_i32, [_i32, ctypes.POINTER(ctypes.c_uint32), _i32]),
    "ctu_convrot_quantize": (_i32, [_vp, _i64, _i64, _i32, _i32, _vp, _vp, _vp]),
    "ctu_convrot_quantize_b128": (_i32, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "ctu_convrot_quantize_staged": (_i32, [_vp, _i64, _i64, _i32, _i32, _i32, _vp, _vp, _vp]),
    "ctu_swiglu_int8_convrot_quantize_scaled": (_i32, [_vp, _i64, _i64, _i32, _vp, _vp, _vp]),
    "ctu_codebook_w4a8_linear": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp]),
    "ctu_codebook_decode_s8": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "ctu_int4_unpack_s8": (_i32, [_vp, _vp, _i64, _i64, _vp]),
    "ctu_convrot_quantize_int4_g128": (_i32, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "ctu_convrot_quantize_int4_g128_b128": (_i32, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "ctu_asym_w4a8_g128_linear": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "ctu_w4a4_g128_linear": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "ctu_int8_linear": (_i32, [_vp, _vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _vp]),
    "ctu_convrot_int8_linear": (_i32, [_vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "ctu_convrot_int8_linear_sync_words": (_i64, [_i64]),
    "ctu_w4a8_linear": (_i32, [_vp, _vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _vp]),
    "ctu_w4a4_linear": (_i32, [_vp, _vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _vp]),
    "ctu_int8_gemm_s32": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "ctu_dequantize_int8_bf16": (_i32, [_vp, _i64, _vp, _vp, _i64, _vp, _i64, _i64, _vp]),
    "ctu_segmented_rms_adaln": (_i32, [_vp, _vp, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _f32, _i32,
                                       _vp]),
    "ctu_layer_norm_adaln": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32, _i32, _vp]),
    "ctu_debug_gemm_injected_timeout": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _u64, _vp]),
    "ctu_debug_set_gemm_kernel": (_i32, [_i32]),
    "ctu_debug_set_fused_linear": (_i32, [_i32]),
    "ctu_debug_set_gemm_split": (_i32, [_i32]),
    "ctu_debug_set_quant_kernel": (_i32, [_i32]),
    "ctu_debug_quant_plan": (_i32, [_i64, _i32, _i32, _i32, _vp, _vp, _vp]),
    "ctu_convrot_w8a8_linear_static_scratch": (_i32, [_vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _vp]),
}


class KernelUnavailable(ImportError):
    """libctu_b200.so is not built or not loadable."""


def library_path() -> Path:
    return _LIB_PATH


def load():
    """Load the CUDA library (once).  Raises KernelUnavailable when it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not _LIB_PATH.exists():
                raise KernelUnavailable(
                    f"{_LIB_PATH} is not built; run comfyui-turing-utils_b200/build.py")
            try:
                lib = ctypes.CDLL(str(_LIB_PATH))
            except OSError as exc:
                raise KernelUnavailable(str(exc)) from exc
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int) -> None:
    """Map a C-ABI status to the exception the reference's pybind layer raises."""
    if rc == CTU_OK:
        return
    msg = load().ctu_last_error().decode(errors="replace")
    # The reference reports contract violations through TORCH_CHECK and CUDA failures
    # through std::runtime_error; both surface in Python as RuntimeError.
    raise RuntimeError(msg or f"libctu_b200 error {rc}")


def device_error(device: int, clear: bool = True) -> int:
    """Read the kernels' bounded-wait error flags for `device` (synchronizes it)."""
    flags = ctypes.c_uint32(0)
    check(load().ctu_get_device_error(int(device), ctypes.byref(flags), 1 if clear else 0))
    return int(flags.value)
