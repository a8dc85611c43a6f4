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
from ._lib_engine import Image, Status

PIXEL_U8, PIXEL_F32_RGB_01 = 0, 1


def vae_tensor_specs(z_dim: int = 48) -> list[tuple[str, tuple[int, ...]]]:
    """The encoder's 82 tensors in the reference's compact GGUF naming
    (weights.cpp:116-167, vae component; artifact.cpp:159): convolutions
    [cout, cin, kh, kw], RMS gains and biases [c]. Mirrors vae_tensor_specs in
    csrc/vae.cu."""
    s: list[tuple[str, tuple[int, ...]]] = []

    def conv(p, co, ci, k):
        s.append((p + ".weight", (co, ci, k, k)))
        s.append((p + ".bias", (co,)))

    def res(p, ci, co):
        s.append((p + ".n1", (ci,)))
        conv(p + ".c1", co, ci, 3)
        s.append((p + ".n2", (co,)))
        conv(p + ".c2", co, co, 3)
        if ci != co:
            conv(p + ".skip", co, ci, 1)

    conv("vae.enc.in", 160, 12, 3)
    cin, cout = (160, 160, 320, 640), (160, 320, 640, 640)
    for b in range(4):
        p = f"vae.enc.down.{b}"
        res(p + ".res.0", cin[b], cout[b])
        res(p + ".res.1", cout[b], cout[b])
        if b < 3:
            conv(p + ".ds", cout[b], cout[b], 3)
    res("vae.enc.mid.res.0", 640, 640)
    s.append(("vae.enc.mid.attn.norm", (640,)))
    conv("vae.enc.mid.attn.qkv", 1920, 640, 1)
    conv("vae.enc.mid.attn.proj", 640, 640, 1)
    res("vae.enc.mid.res.1", 640, 640)
    s.append(("vae.enc.out_norm", (640,)))
    conv("vae.enc.out", 2 * z_dim, 640, 3)
    conv("vae.quant", 2 * z_dim, 2 * z_dim, 1)
    return s


def vae_synthetic_stats(z_dim: int = 48):
    """Latent mean / std of the synthetic encoder (csrc/vae.cu load_weights)."""
    c = np.arange(z_dim, dtype=np.float32)
    return (np.float32(0.05) * np.sin(c)).astype(np.float32), (np.float32(0.5) + np.float32(0.01) * c).astype(np.float32)


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


class VaeOptions(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("artifact_path", C.c_char_p),
                ("synthetic_seed", C.c_uint64), ("image_width", C.c_int),
                ("image_height", C.c_int), ("z_dim", C.c_int), ("device_index", C.c_int),
                ("use_cuda_graph", C.c_int)]


def _attach_vae(lib):
    if getattr(lib, "_vae_sigs", False):
        return lib
    _attach(lib)
    st = C.POINTER(Status)
    vp = C.c_void_p
    lib.wam_b200_vae_create.restype = C.c_int
    lib.wam_b200_vae_create.argtypes = [C.POINTER(VaeOptions), C.POINTER(vp), st]
    lib.wam_b200_vae_destroy.restype = None
    lib.wam_b200_vae_destroy.argtypes = [vp]
    lib.wam_b200_vae_info.restype = C.c_int
    lib.wam_b200_vae_info.argtypes = [vp, C.POINTER(C.c_int), C.POINTER(C.c_int),
                                      C.POINTER(C.c_double)]
    lib.wam_b200_vae_encode.restype = C.c_int
    lib.wam_b200_vae_encode.argtypes = [vp, C.POINTER(Image), C.c_int, C.POINTER(C.c_float),
                                        C.c_size_t, st]
    lib.wam_b200_vae_encode_device.restype = C.c_int
    lib.wam_b200_vae_encode_device.argtypes = [vp, vp, vp, vp, st]
    lib.wam_b200_vae_read_stage.restype = C.c_int
    lib.wam_b200_vae_read_stage.argtypes = [vp, C.c_char_p, C.POINTER(C.c_float), C.c_size_t,
                                            C.POINTER(C.c_int), C.POINTER(C.c_int),
                                            C.POINTER(C.c_int)]
    lib._vae_sigs = True
    return lib


class Vae:
    """The Wan VAE encoder (run_vae, src/models/gwp05/engine/vae.cpp:279-388):
    three camera views -> standardised latent [z][H/16][W/16]."""

    def __init__(self, width: int, height: int, z_dim: int = 48, seed: int = 0,
                 artifact: str | None = None, device_index: int = 0, graphs: bool = True):
        self.lib = _attach_vae(load())
        o = VaeOptions(C.sizeof(VaeOptions), artifact.encode() if artifact else None, seed, width,
                       height, z_dim, device_index, 1 if graphs else 0)
        self.h = C.c_void_p()
        st = Status()
        _raise(self.lib, self.lib.wam_b200_vae_create(C.byref(o), C.byref(self.h), C.byref(st)),
               st, "wam_b200_vae_create")
        self.width, self.height, self.z = width, height, z_dim
        n, l, f = C.c_int(), C.c_int(), C.c_double()
        self.lib.wam_b200_vae_info(self.h, C.byref(n), C.byref(l), C.byref(f))
        self.latent_count, self.launches, self.flops = n.value, l.value, f.value

    def encode(self, views) -> np.ndarray:
        """Host views (uint8 / float32 HWC RGB) -> host latent [z, H/16, W/16]."""
        views = [np.ascontiguousarray(v) for v in views]
        out = np.zeros((self.z, self.height // 16, self.width // 16), np.float32)
        st = Status()
        _raise(self.lib, self.lib.wam_b200_vae_encode(
            self.h, _images(views, lambda v: v.ctypes.data), len(views),
            out.ctypes.data_as(C.POINTER(C.c_float)), out.size, C.byref(st)),
               st, "wam_b200_vae_encode")
        return out

    def encode_device(self, pixels: torch.Tensor, latent: torch.Tensor | None = None):
        """Device pixels [12, H/2, W/2] F32 -> device latent (current stream)."""
        if latent is None:
            latent = torch.empty((self.z, self.height // 16, self.width // 16),
                                 dtype=torch.float32, device=pixels.device)
        st = Status()
        _raise(self.lib, self.lib.wam_b200_vae_encode_device(
            self.h, C.c_void_p(pixels.data_ptr()), C.c_void_p(latent.data_ptr()),
            C.c_void_p(torch.cuda.current_stream().cuda_stream), C.byref(st)),
               st, "wam_b200_vae_encode_device")
        return latent

    def stage(self, name: str) -> np.ndarray:
        """An intermediate NHWC activation of the last encode, as F32 [H, W, C]."""
        h, w, c = C.c_int(), C.c_int(), C.c_int()
        buf = np.zeros(self.height * self.width * 160 // 4 + 1, np.float32)
        rc = self.lib.wam_b200_vae_read_stage(self.h, name.encode(),
                                              buf.ctypes.data_as(C.POINTER(C.c_float)), buf.size,
                                              C.byref(h), C.byref(w), C.byref(c))
        if rc != 0:
            raise RuntimeError(f"wam_b200_vae_read_stage({name}) failed: "
                               f"{self.lib.wam_b200_last_error().decode()}")
        return buf[:h.value * w.value * c.value].reshape(h.value, w.value, c.value)

    def close(self):
        if self.h:
            self.lib.wam_b200_vae_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
