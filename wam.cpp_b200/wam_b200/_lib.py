"""ctypes loader for libwam_b200.so (the engine's C ABI, include/wam_b200.h).

The library is built in-tree by wam.cpp_b200/build.py (WAM_B200_LIB names
another build of it). Loading fails loudly if it is missing: there is no
fallback implementation of any entry point.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = PKG_ROOT / "lib" / "libwam_b200.so"

_lib = None

vp = C.c_void_p
i32 = C.c_int
f32p = C.POINTER(C.c_float)
u32p = C.POINTER(C.c_uint)
sz = C.c_size_t


def _sig(lib, name, restype, argtypes):
    fn = getattr(lib, name)
    fn.restype = restype
    fn.argtypes = argtypes
    return fn


def load(path: Path | None = None):
    """Loads (once) and returns the library with prototypes attached."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else Path(os.environ.get("WAM_B200_LIB", LIB_PATH))
    if not p.exists():
        raise RuntimeError(f"libwam_b200.so not built ({p}); run python wam.cpp_b200/build.py")
    lib = C.CDLL(str(p))
    _sig(lib, "wam_b200_abi_version", C.c_uint32, [])
    _sig(lib, "wam_b200_last_error", C.c_char_p, [])
    _sig(lib, "wam_b200_gemm_scratch_floats", sz, [i32, i32, i32, i32, C.POINTER(i32)])
    _sig(lib, "wam_b200_op_gemm", i32,
         [vp, i32, i32, vp, i32, i32, i32, vp, vp, vp, i32, vp, i32, vp, sz, vp, i32, vp, i32, vp])
    _sig(lib, "wam_b200_op_gemm_noalloc", i32,
         [vp, i32, i32, vp, i32, i32, i32, vp, vp, vp, i32, vp, i32, i32, vp])
    _sig(lib, "wam_b200_op_gemm_noalloc_error", i32, [u32p])
    _sig(lib, "wam_b200_op_retile_weights", i32, [vp, vp, i32, i32, vp])
    _sig(lib, "wam_b200_op_q8_quantize", i32, [vp, C.c_longlong, vp, vp])
    _sig(lib, "wam_b200_op_q8_retile", i32, [vp, vp, i32, i32, vp])
    _sig(lib, "wam_b200_op_attention", i32,
         [vp, C.c_longlong, C.c_longlong, vp, vp, C.c_longlong, C.c_longlong, i32, i32, i32, i32,
          C.c_float, vp, i32, vp])
    _sig(lib, "wam_b200_op_layernorm", i32, [vp, i32, i32, vp, vp, C.c_float, i32, vp, vp])
    _sig(lib, "wam_b200_op_qkv_scatter", i32, [vp, vp])
    _sig(lib, "wam_b200_rope_inv_freq", i32, [i32, C.POINTER(C.c_float)])
    _sig(lib, "wam_b200_op_synth", i32, [vp, C.c_longlong, C.c_uint64, C.c_double, C.c_double, vp])
    _sig(lib, "wam_b200_tensor_seed", C.c_uint64, [C.c_uint64, C.c_char_p])
    f32p = C.POINTER(C.c_float)
    _sig(lib, "wam_b200_flow_schedule", i32, [i32, C.c_float, f32p, f32p])
    _sig(lib, "wam_b200_visual_positions", i32, [i32, i32, C.POINTER(C.c_int)])
    _sig(lib, "wam_b200_normalize_state", i32, [f32p, i32, i32, f32p, f32p, f32p])
    _sig(lib, "wam_b200_postprocess_action", i32, [f32p, i32, i32, i32, f32p, f32p, f32p, f32p])
    from . import _lib_engine
    _lib_engine.attach(lib, _sig)
    _lib = lib
    return lib


def last_error() -> str:
    return load().wam_b200_last_error().decode()


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed (code {rc}): {last_error()}")
