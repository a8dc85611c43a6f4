"""CPU oracle of the GWP-0.5 MoT forward pass — TEST INFRASTRUCTURE ONLY.

Loaded only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
legs, always as the checker (or the timed CPU baseline), never by the product
path. See oracle.h for what it restates and its parity status.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

from .synth import Geometry, Request, make_weights, statistics  # noqa: F401

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libwamref.so"


class _Geom(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "hidden", "layers", "heads", "ffn", "action_hidden", "action_ffn", "action_dim",
        "real_state_dim", "real_action_dim", "num_embodiments", "embodiment_id", "grid_h",
        "grid_w", "vae_z", "action_chunk", "steps", "prompt_tokens", "text_dim")] + [
        ("norm_eps", C.c_float), ("flow_shift", C.c_float)]


def geom_struct(g: Geometry, cls=_Geom):
    s = cls()
    for name, _ in cls._fields_:
        setattr(s, name, getattr(g, name))
    return s


def reference_root() -> Path | None:
    """The reference source tree named by WAM_REFERENCE_ROOT, if it holds the
    host sources the _ref build compiles (None otherwise)."""
    root = os.environ.get("WAM_REFERENCE_ROOT")
    if root and (Path(root) / "src" / "models" / "common" / "scheduler.cpp").exists():
        return Path(root)
    return None


def build(with_ref: bool = True) -> None:
    """Builds liboracle.so (and, when WAM_REFERENCE_ROOT names the reference
    tree, the reference's own scheduler/semantics into _ref/libwamref.so)."""
    subprocess.run(["make", "-C", str(HERE), "liboracle.so"], check=True, capture_output=True)
    ref = reference_root()
    if with_ref and ref is not None:
        subprocess.run(["make", "-C", str(HERE), "ref", f"REF={ref}"], check=True,
                       capture_output=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build(with_ref=False)
        l = C.CDLL(str(LIB))
        f32p = C.POINTER(C.c_float)
        l.oracle_create.restype = C.c_void_p
        l.oracle_create.argtypes = [C.POINTER(_Geom), C.c_int, C.POINTER(C.c_char_p),
                                    C.POINTER(C.c_void_p), C.POINTER(C.c_int64), f32p, f32p,
                                    f32p, f32p, C.c_char_p, C.c_int]
        l.oracle_destroy.argtypes = [C.c_void_p]
        l.oracle_create_synthetic.restype = C.c_void_p
        l.oracle_create_synthetic.argtypes = [C.POINTER(_Geom), C.c_uint64, C.c_double, C.c_char_p,
                                              C.c_int]
        l.oracle_predict.restype = C.c_int
        l.oracle_predict.argtypes = [C.c_void_p] + [f32p] * 10
        l.oracle_schedule.argtypes = [C.c_int, C.c_float, f32p, f32p]
        l.oracle_timestep_embedding.argtypes = [C.c_float, C.c_int, f32p]
        l.oracle_visual_positions.argtypes = [C.c_int, C.c_int] + [C.POINTER(C.c_int32)] * 3
        l.oracle_threads.restype = C.c_int
        l.oracle_quantize_q8.argtypes = [C.c_void_p]
        l.oracle_q8_roundtrip.argtypes = [C.c_void_p, C.c_int64, f32p]
        l.oracle_set_uncached.argtypes = [C.c_void_p, C.c_int]
        l.oracle_create_synthetic_ex.restype = C.c_void_p
        l.oracle_create_synthetic_ex.argtypes = [C.POINTER(_Geom), C.c_uint64, C.c_double, C.c_int,
                                                 C.c_char_p, C.c_int]
        l.oracle_block.restype = C.c_int
        l.oracle_block.argtypes = [C.c_void_p, C.c_int, C.c_float] + [f32p] * 6
        i32p = C.POINTER(C.c_int)
        l.oracle_t5_encode.restype = C.c_int
        l.oracle_t5_encode.argtypes = [C.POINTER(C.c_char_p), C.POINTER(C.c_void_p), C.c_int,
                                       C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                       C.POINTER(C.c_int32), C.c_int, C.c_int, f32p]
        l.oracle_vae_encode.restype = C.c_int
        l.oracle_vae_encode.argtypes = [C.POINTER(C.c_char_p), C.POINTER(C.c_void_p), C.c_int,
                                        f32p, f32p, C.c_int, f32p, C.c_int, C.c_int, f32p,
                                        C.c_char_p, f32p, i32p]
        l.oracle_compose_and_patchify.restype = C.c_int
        l.oracle_compose_and_patchify.argtypes = [C.POINTER(C.c_void_p), i32p, i32p, i32p,
                                                  C.c_int, C.c_int, f32p]
        _lib = l
    return _lib


def ref_lib():
    """The reference's own scheduler.cpp/semantics.cpp (None if not built)."""
    if not REF_LIB.exists():
        return None
    l = C.CDLL(str(REF_LIB))
    f32p = C.POINTER(C.c_float)
    i32p = C.POINTER(C.c_int32)
    l.wamref_schedule.argtypes = [C.c_int, C.c_float, f32p, f32p]
    l.wamref_visual_positions.argtypes = [C.c_int, C.c_int, i32p, i32p, i32p]
    l.wamref_action_positions.argtypes = [C.c_int, C.c_int, i32p]
    l.wamref_normalize_state.argtypes = [f32p, C.c_int, C.c_int, f32p, f32p, f32p]
    l.wamref_postprocess.argtypes = [f32p, C.c_int, C.c_int, C.c_int, f32p, f32p, f32p, C.c_int, f32p]
    return l


REF_VISION_LIB = REF_LIB.parent / "libwamref_vision.so"


def _views_args(views):
    data = (C.c_void_p * 3)(*[v.ctypes.data for v in views])
    ints = lambda xs: (C.c_int * 3)(*xs)  # noqa: E731
    return (data, ints([v.shape[1] for v in views]), ints([v.shape[0] for v in views]),
            ints([0 if v.dtype == np.uint8 else 1 for v in views]))


def compose_and_patchify(views, out_w: int, out_h: int, reference: bool = False) -> np.ndarray:
    """Vision stage 1 on three HWC RGB views (uint8, or float32 in [0, 1]):
    [12][out_h/2][out_w/2] float32. reference=True runs the reference's own
    compose_and_patchify (oracle/_ref/libwamref_vision.so, `make ref`)."""
    views = [np.ascontiguousarray(v) for v in views]
    out = np.zeros((12, out_h // 2, out_w // 2), np.float32)
    d, w, h, f = _views_args(views)
    if reference:
        if not REF_VISION_LIB.exists():
            raise FileNotFoundError(REF_VISION_LIB)
        rl = C.CDLL(str(REF_VISION_LIB))
        rl.wamref_compose_and_patchify.restype = C.c_int
        rc = rl.wamref_compose_and_patchify(d, w, h, f, out_w, out_h, _fp(out), C.c_longlong(out.size))
    else:
        rc = lib().oracle_compose_and_patchify(d, w, h, f, out_w, out_h, _fp(out))
    if rc != 0:
        raise ValueError("compose_and_patchify rejected its inputs")
    return out


def t5_encode(weights: dict, g, tokens, max_tokens: int):
    """UMT5 encoder (oracle/t5.cpp): tokens [n] -> [max_tokens][hidden] F32.
    g: wam_b200.text.T5Geometry-like (hidden, heads, head_dim, ffn, layers, vocab)."""
    names = list(weights)
    arrs = [np.ascontiguousarray(weights[n], dtype=np.uint16) for n in names]
    cn = (C.c_char_p * len(names))(*[n.encode() for n in names])
    ct = (C.c_void_p * len(names))(*[a.ctypes.data for a in arrs])
    tok = np.ascontiguousarray(tokens, np.int32)
    out = np.zeros((max_tokens, g.hidden), np.float32)
    rc = lib().oracle_t5_encode(cn, ct, len(names), g.hidden, g.heads, g.head_dim, g.ffn, g.layers,
                                g.vocab, tok.ctypes.data_as(C.POINTER(C.c_int32)), tok.size,
                                max_tokens, _fp(out))
    if rc != 0:
        raise ValueError(f"oracle_t5_encode failed ({rc})")
    return out


def vae_encode(weights: dict, mean, std, z: int, pixels, width: int, height: int,
               stage: str | None = None):
    """Wan VAE encoder (oracle/vae.cpp) on stage-1 pixels [12][H/2][W/2]:
    latent [z][H/16][W/16] (and the NHWC activation named by `stage`)."""
    names = list(weights)
    arrs = [np.ascontiguousarray(weights[n], dtype=np.uint16) for n in names]
    cn = (C.c_char_p * len(names))(*[n.encode() for n in names])
    ct = (C.c_void_p * len(names))(*[a.ctypes.data for a in arrs])
    mean = np.ascontiguousarray(mean, np.float32)
    std = np.ascontiguousarray(std, np.float32)
    pixels = np.ascontiguousarray(pixels, np.float32)
    lat = np.zeros((z, height // 16, width // 16), np.float32)
    st = np.zeros(height * width * 160 // 4 + 1, np.float32) if stage else None
    dims = (C.c_int * 3)()
    rc = lib().oracle_vae_encode(cn, ct, len(names), _fp(mean), _fp(std), z, _fp(pixels), width,
                                 height, _fp(lat), stage.encode() if stage else None,
                                 _fp(st) if stage else None, dims)
    if rc != 0:
        raise ValueError(f"oracle_vae_encode failed ({rc})")
    if stage:
        return lat, st[:dims[0] * dims[1] * dims[2]].reshape(dims[0], dims[1], dims[2])
    return lat


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float)) if a is not None else None


def schedule(steps: int, shift: float):
    ts = np.zeros(steps, np.float32)
    sig = np.zeros(steps + 1, np.float32)
    lib().oracle_schedule(steps, shift, _fp(ts), _fp(sig))
    return ts, sig


def q8_roundtrip(bf16_bits: np.ndarray) -> np.ndarray:
    """GGML Q8_0 quantise + dequantise (F32 q * d) of BF16 bit patterns."""
    b = np.ascontiguousarray(bf16_bits, dtype=np.uint16).reshape(-1)
    out = np.zeros(b.size, np.float32)
    lib().oracle_q8_roundtrip(b.ctypes.data, b.size, _fp(out))
    return out


def timestep_embedding(t: float, dim: int = 256):
    out = np.zeros(dim, np.float32)
    lib().oracle_timestep_embedding(t, dim, _fp(out))
    return out


class OracleModel:
    """A CPU model over BF16 weights given as {compact name: uint16 array}."""

    def __init__(self, g: Geometry, weights: dict | None, stats: dict | None = None,
                 seed: int = 0, bias_scale: float = 0.0, ffn_kind: int = 0):
        """weights None: the synthetic weights of (seed, bias_scale), built in C++
        (ffn_kind 1: SiLU-gated FFN weights, the config-1 variant)."""
        self.g = g
        if weights is None:
            err = C.create_string_buffer(512)
            gs = geom_struct(g)
            self.h = lib().oracle_create_synthetic_ex(C.byref(gs), seed, bias_scale, ffn_kind, err,
                                                      512)
            if not self.h:
                raise RuntimeError("oracle_create_synthetic: " + err.value.decode())
            return
        stats = stats or statistics(g)
        names = list(weights)
        arrs = [np.ascontiguousarray(weights[n], dtype=np.uint16) for n in names]
        cn = (C.c_char_p * len(names))(*[n.encode() for n in names])
        cd = (C.c_void_p * len(names))(*[a.ctypes.data for a in arrs])
        ce = (C.c_int64 * len(names))(*[a.size for a in arrs])
        err = C.create_string_buffer(512)
        self._stats = {k: np.ascontiguousarray(v, np.float32) for k, v in stats.items()}
        gs = geom_struct(g)
        self.h = lib().oracle_create(C.byref(gs), len(names), cn, cd, ce,
                                     _fp(self._stats["state_q01"]), _fp(self._stats["state_q99"]),
                                     _fp(self._stats["action_q01"]), _fp(self._stats["action_q99"]),
                                     err, 512)
        if not self.h:
            raise RuntimeError("oracle_create: " + err.value.decode())

    def quantize_q8(self) -> "OracleModel":
        """Config 5: linear weights become their exact F32 Q8_0 dequantisation."""
        lib().oracle_quantize_q8(self.h)
        return self

    def set_uncached(self, uncached: bool = True) -> "OracleModel":
        """Recompute the prefix every step (the reference's CPU mode)."""
        lib().oracle_set_uncached(self.h, 1 if uncached else 0)
        return self

    def block(self, t: float, xv, xa, tv, ta, norm_kind: int = 0):
        """Config 1: one MoT layer over given hidden states (oracle_block).
        xv [V, H], xa [1 + T, E] (state row first), tv [Nt, H], ta [Nt, E].
        Returns (visual out [V, H], action stream out [1 + T, E])."""
        g = self.g
        args = [np.ascontiguousarray(a, np.float32) for a in (xv, xa, tv, ta)]
        ov = np.zeros((g.visual_tokens, g.hidden), np.float32)
        oa = np.zeros((1 + g.action_chunk, g.action_hidden), np.float32)
        rc = lib().oracle_block(self.h, norm_kind, t, *[_fp(a) for a in args], _fp(ov), _fp(oa))
        if rc != 0:
            raise RuntimeError("oracle_block failed")
        return ov, oa

    def __del__(self):
        h = getattr(self, "h", None)
        if h:
            lib().oracle_destroy(h)
            self.h = None

    def predict(self, req: Request, dumps: bool = False) -> dict:
        g = self.g
        P, L, Hd, Nt = g.prefix_tokens, g.layers, g.heads, g.prompt_tokens
        out = np.zeros((g.action_chunk, g.real_action_dim), np.float32)
        d = {}
        if dumps:
            d = {"prefix_k": np.zeros((L, Hd, P, 128), np.float32),
                 "prefix_v": np.zeros((L, Hd, P, 128), np.float32),
                 "prompt_k": np.zeros((L, Hd, Nt, 128), np.float32),
                 "prompt_v": np.zeros((L, Hd, Nt, 128), np.float32),
                 "velocity": np.zeros((g.steps, g.action_chunk, g.action_dim), np.float32),
                 "actions": np.zeros((g.steps, g.action_chunk, g.action_dim), np.float32)}
        args = [np.ascontiguousarray(a, np.float32) for a in (req.state, req.latent, req.prompt, req.noise)]
        rc = lib().oracle_predict(self.h, *[_fp(a) for a in args], _fp(out),
                                  *[_fp(d.get(k)) for k in ("prefix_k", "prefix_v", "prompt_k",
                                                            "prompt_v", "velocity", "actions")])
        if rc != 0:
            raise RuntimeError("oracle_predict failed")
        d["action"] = out
        return d
