"""UMT5 text encoder of the engine (the step before the prompt cache when the
language encoder is resident), over the C ABI's wam_b200_t5_* entry points:
prompt token ids -> prompt embedding [max_tokens, hidden] F32, the reference's
run_t5 (src/models/gwp05/engine/text_encoder.cpp:112-204)."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import load
from ._lib_engine import Status


@dataclass(frozen=True)
class T5Geometry:
    vocab: int = 256384
    hidden: int = 4096
    ffn: int = 10240
    heads: int = 64
    head_dim: int = 64
    layers: int = 24
    max_tokens: int = 512


# UMT5-XXL as used by GWP-0.5 (gwp05.t5_* keys) and a small parity geometry.
T5_XXL = T5Geometry()
T5_TINY = T5Geometry(vocab=1000, hidden=256, ffn=512, heads=4, head_dim=64, layers=2,
                     max_tokens=64)


def t5_tensor_specs(g: T5Geometry) -> list[tuple[str, tuple[int, ...]]]:
    """The encoder's tensors in the reference's compact naming (weights.cpp:146-153,
    t5 component): 2 + 10 per layer (gwp05_gguf.py component_expected_counts).
    Mirrors t5_tensor_specs in csrc/t5.cu."""
    H, I, F = g.hidden, g.heads * g.head_dim, g.ffn
    s = [("t5.token_embd.weight", (g.vocab, H))]
    for layer in range(g.layers):
        p = f"t5.blk.{layer}"
        s += [(p + ".sa.q.weight", (I, H)), (p + ".sa.k.weight", (I, H)),
              (p + ".sa.v.weight", (I, H)), (p + ".sa.o.weight", (H, I)),
              (p + ".sa.rel.weight", (32, g.heads)), (p + ".sa_norm.weight", (H,)),
              (p + ".ffn.wi0.weight", (F, H)), (p + ".ffn.wi1.weight", (F, H)),
              (p + ".ffn.wo.weight", (H, F)), (p + ".ffn_norm.weight", (H,))]
    s.append(("t5.final_norm.weight", (H,)))
    return s


class T5Options(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("artifact_path", C.c_char_p),
                ("synthetic_seed", C.c_uint64), ("vocab", C.c_int), ("hidden", C.c_int),
                ("ffn", C.c_int), ("heads", C.c_int), ("head_dim", C.c_int), ("layers", C.c_int),
                ("max_tokens", C.c_int), ("device_index", C.c_int), ("use_cuda_graphs", C.c_int)]


def _attach(lib):
    if getattr(lib, "_t5_sigs", False):
        return lib
    st = C.POINTER(Status)
    vp, i32 = C.c_void_p, C.c_int
    i32p = C.POINTER(C.c_int32)
    lib.wam_b200_t5_create.restype = i32
    lib.wam_b200_t5_create.argtypes = [C.POINTER(T5Options), C.POINTER(vp), st]
    lib.wam_b200_t5_destroy.restype = None
    lib.wam_b200_t5_destroy.argtypes = [vp]
    lib.wam_b200_t5_geometry.restype = i32
    lib.wam_b200_t5_geometry.argtypes = [vp] + [C.POINTER(i32)] * 6
    lib.wam_b200_t5_encode.restype = i32
    lib.wam_b200_t5_encode.argtypes = [vp, i32p, i32, i32p, i32, C.POINTER(C.c_float), C.c_size_t, st]
    lib.wam_b200_t5_encode_device.restype = i32
    lib.wam_b200_t5_encode_device.argtypes = [vp, i32p, i32, i32p, i32, vp, vp, st]
    lib.wam_b200_t5_info.restype = i32
    lib.wam_b200_t5_info.argtypes = [vp, i32, C.POINTER(C.c_double), C.POINTER(i32)]
    lib.wam_b200_t5_relative_bucket.restype = i32
    lib.wam_b200_t5_relative_bucket.argtypes = [i32, i32, i32]
    lib._t5_sigs = True
    return lib


def relative_bucket(relative: int, buckets: int = 32, max_distance: int = 128) -> int:
    return _attach(load()).wam_b200_t5_relative_bucket(relative, buckets, max_distance)


def _raise(lib, rc, st, what):
    if rc != 0:
        msg = C.string_at(st.message).decode() if st.message else "?"
        lib.wam_b200_status_free(C.byref(st))
        raise RuntimeError(f"{what} failed (code {rc}): {msg}")


class TextEncoder:
    def __init__(self, geometry: T5Geometry = T5_XXL, seed: int = 0, artifact: str | None = None,
                 device_index: int = 0, graphs: bool = True):
        self.lib = _attach(load())
        g = geometry
        o = T5Options(C.sizeof(T5Options), artifact.encode() if artifact else None, seed, g.vocab,
                      g.hidden, g.ffn, g.heads, g.head_dim, g.layers, g.max_tokens, device_index,
                      1 if graphs else 0)
        self.h = C.c_void_p()
        st = Status()
        _raise(self.lib, self.lib.wam_b200_t5_create(C.byref(o), C.byref(self.h), C.byref(st)),
               st, "wam_b200_t5_create")
        vals = [C.c_int() for _ in range(6)]
        self.lib.wam_b200_t5_geometry(self.h, *[C.byref(v) for v in vals])
        self.geometry = T5Geometry(vals[0].value, vals[1].value, vals[2].value, vals[3].value, 64,
                                   vals[4].value, vals[5].value)

    def encode(self, tokens, mask=None) -> np.ndarray:
        tok = np.ascontiguousarray(tokens, np.int32)
        m = None if mask is None else np.ascontiguousarray(mask, np.int32)
        g = self.geometry
        out = np.zeros((g.max_tokens, g.hidden), np.float32)
        st = Status()
        i32p = C.POINTER(C.c_int32)
        _raise(self.lib, self.lib.wam_b200_t5_encode(
            self.h, tok.ctypes.data_as(i32p), tok.size,
            m.ctypes.data_as(i32p) if m is not None else None, 0 if m is None else m.size,
            out.ctypes.data_as(C.POINTER(C.c_float)), out.size, C.byref(st)),
               st, "wam_b200_t5_encode")
        return out

    def encode_device(self, tokens, out: torch.Tensor | None = None) -> torch.Tensor:
        g = self.geometry
        tok = np.ascontiguousarray(tokens, np.int32)
        if out is None:
            out = torch.empty((g.max_tokens, g.hidden), dtype=torch.float32, device="cuda")
        st = Status()
        _raise(self.lib, self.lib.wam_b200_t5_encode_device(
            self.h, tok.ctypes.data_as(C.POINTER(C.c_int32)), tok.size, None, 0,
            C.c_void_p(out.data_ptr()), C.c_void_p(torch.cuda.current_stream().cuda_stream),
            C.byref(st)), st, "wam_b200_t5_encode_device")
        return out

    def info(self, n: int):
        f, l = C.c_double(), C.c_int()
        self.lib.wam_b200_t5_info(self.h, n, C.byref(f), C.byref(l))
        return f.value, l.value

    def close(self):
        if self.h:
            self.lib.wam_b200_t5_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
