"""Vision front-end of the engine (the step before the prefix when raw camera
images arrive), over the C ABI's vision entry points.

Stage 1, ``Preprocessor`` / ``preprocess``: three views composed onto the
image canvas, resized to cover each cell (triangle filter, centre crop),
patchified 2x2 into [12][H/2][W/2] F32 in [-1, 1] -- the reference's
compose_and_patchify (src/models/gwp05/engine/vae.cpp:1-134) and its CUDA
preprocessor (src/models/gwp05/kernels/cuda_preprocess.{h,cu}), bit for bit
with the former.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import load
from ._lib_engine import Status

PIXEL_U8, PIXEL_F32_RGB_01 = 0, 1


class Image(C.Structure):
    _fields_ = [("data", C.c_void_p), ("w", C.c_int), ("h", C.c_int), ("format", C.c_int)]


def _attach(lib):
    if getattr(lib, "_vision_sigs", False):
        return lib
    st = C.POINTER(Status)
    lib.wam_b200_preprocessor_create.restype = C.c_int
    lib.wam_b200_preprocessor_create.argtypes = [C.c_int, C.POINTER(C.c_void_p), st]
    lib.wam_b200_preprocessor_destroy.restype = None
    lib.wam_b200_preprocessor_destroy.argtypes = [C.c_void_p]
    lib.wam_b200_preprocess.restype = C.c_int
    lib.wam_b200_preprocess.argtypes = [C.c_void_p, C.POINTER(Image), C.c_int, C.c_int, C.c_int,
                                        C.c_void_p, C.c_void_p, st]
    lib.wam_b200_op_preprocess.restype = C.c_int
    lib.wam_b200_op_preprocess.argtypes = [C.POINTER(Image), C.c_int, C.c_int, C.c_void_p,
                                           C.c_void_p]
    lib._vision_sigs = True
    return lib


def _format(dtype) -> int:
    if dtype in (np.uint8, torch.uint8):
        return PIXEL_U8
    if dtype in (np.float32, torch.float32):
        return PIXEL_F32_RGB_01
    raise ValueError(f"views must be uint8 or float32 HWC RGB, got {dtype}")


def _images(views, ptr):
    arr = (Image * len(views))()
    for i, v in enumerate(views):
        if v.ndim != 3 or v.shape[2] != 3:
            raise ValueError("views must be HWC RGB arrays")
        arr[i] = Image(ptr(v), int(v.shape[1]), int(v.shape[0]), _format(v.dtype))
    return arr


def _raise(lib, rc, st, what):
    if rc != 0:
        msg = C.string_at(st.message).decode() if st.message else "?"
        lib.wam_b200_status_free(C.byref(st))
        raise RuntimeError(f"{what} failed (code {rc}): {msg}")


class Preprocessor:
    """gwp05_cuda_preprocessor_{create,destroy} + gwp05_cuda_preprocess:
    host views in, device canvas out (the call returns once it is written)."""

    def __init__(self, device_index: int = 0):
        self.lib = _attach(load())
        self.h = C.c_void_p()
        st = Status()
        _raise(self.lib, self.lib.wam_b200_preprocessor_create(device_index, C.byref(self.h),
                                                               C.byref(st)),
               st, "wam_b200_preprocessor_create")
        self.device = torch.device("cuda", device_index)

    def __call__(self, views, width: int, height: int, out=None) -> torch.Tensor:
        views = [np.ascontiguousarray(v) for v in views]
        if out is None:
            out = torch.empty((12, height // 2, width // 2), dtype=torch.float32,
                              device=self.device)
        imgs = _images(views, lambda v: v.ctypes.data)
        st = Status()
        stream = C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        _raise(self.lib, self.lib.wam_b200_preprocess(self.h, imgs, len(views), width, height,
                                                      C.c_void_p(out.data_ptr()), stream,
                                                      C.byref(st)),
               st, "wam_b200_preprocess")
        return out

    def close(self):
        if self.h:
            self.lib.wam_b200_preprocessor_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def preprocess(views, width: int, height: int, out=None) -> torch.Tensor:
    """The same kernel on three views already on the device (uint8 or float32
    HWC RGB CUDA tensors), asynchronous on the current stream."""
    lib = _attach(load())
    views = [v.contiguous() for v in views]
    if out is None:
        out = torch.empty((12, height // 2, width // 2), dtype=torch.float32,
                          device=views[0].device)
    imgs = _images(views, lambda v: v.data_ptr())
    rc = lib.wam_b200_op_preprocess(imgs, width, height, C.c_void_p(out.data_ptr()),
                                    C.c_void_p(torch.cuda.current_stream().cuda_stream))
    if rc != 0:
        raise RuntimeError(f"wam_b200_op_preprocess failed (code {rc}): "
                           f"{lib.wam_b200_last_error().decode()}")
    return out
