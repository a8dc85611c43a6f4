"""Host-side mirror of the reference's engine boundary over the wam_b200 C ABI.

Engine mirrors wam::internal::gwp05::engine::Engine
(src/models/gwp05/engine/engine.h:142-155): predict() returns the de-normalised
action chunk for one request and raises on failure (the reference returns an
empty vector that the model layer maps to inference_failed); reset() drops the
projected-prompt cache. predict_batch() adds the batched entry the reference
lacks.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import load
from ._lib_engine import (Image, GEOM_FIELDS, BlockInputs, Geometry, GraphProfile, OpProfile, Options,
                          Request, Stats, Status)

KINDS = ("gemm", "attention", "layernorm", "qkv_scatter", "small_linear", "elementwise", "sync")
PHASES = ("prompt", "prefix", "denoise")


class EngineError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


def _raise(lib, rc, st, what):
    if rc != 0:
        msg = C.cast(st.message, C.c_char_p).value.decode() if st.message else ""
        lib.wam_b200_status_free(C.byref(st))
        raise EngineError(rc, f"{what}: {msg}")


def geometry_struct(g) -> Geometry:
    s = Geometry()
    for n in GEOM_FIELDS:
        setattr(s, n, int(getattr(g, n)))
    s.norm_eps = float(g.norm_eps)
    s.flow_shift = float(g.flow_shift)
    return s


@dataclass
class Req:
    """One request. `latent` is the precomputed VAE latent; with latent None,
    `images` (three HWC RGB views, uint8 or float32) run the engine's vision
    front-end (engine created with vae=True). `prompt` is the precomputed
    prompt embedding; with prompt None, `tokens` (and an optional 0/1 `mask`)
    run the UMT5 encoder (engine created with t5=True)."""
    state: np.ndarray
    latent: np.ndarray | None
    prompt: np.ndarray | None
    noise: np.ndarray | None = None
    images: list | None = None
    tokens: np.ndarray | None = None  # prompt token ids (engine created with t5=True)
    mask: np.ndarray | None = None


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class Engine:
    def __init__(self, geometry=None, seed: int = 0, artifact: str | None = None,
                 bias_scale: float = 0.0, device: int = 0, max_batch: int = 1,
                 graphs: bool = True, prompt_cache: bool = True, weights: str = "bf16",
                 ffn: str = "gelu", norm: str = "layernorm", block: bool = False,
                 vae: bool = False, t5: bool = False, t5_vocab: int = 0, t5_ffn: int = 0,
                 t5_layers: int = 0):
        """ffn ('gelu' | 'swiglu') and norm ('layernorm' | 'rmsnorm') select the
        config-1 block variants (synthetic weights); block=True creates an engine
        for block_forward (one layer over given hidden states)."""
        self.lib = load()
        o = Options()
        o.struct_size = C.sizeof(Options)
        o.artifact_path = artifact.encode() if artifact else None
        if geometry is not None:
            o.synthetic_geometry = geometry_struct(geometry)
        o.synthetic_seed = seed
        o.synthetic_bias_scale = bias_scale
        o.device_index = device
        o.max_batch = max_batch
        o.use_cuda_graphs = 1 if graphs else 0
        o.prompt_cache = 1 if prompt_cache else 0
        if weights not in ("bf16", "q8_0"):
            raise ValueError("weights must be 'bf16' or 'q8_0'")
        o.weight_format = 1 if weights == "q8_0" else 0
        if ffn not in ("gelu", "swiglu") or norm not in ("layernorm", "rmsnorm"):
            raise ValueError("ffn must be 'gelu' or 'swiglu', norm 'layernorm' or 'rmsnorm'")
        o.ffn_kind = 1 if ffn == "swiglu" else 0
        o.norm_kind = 1 if norm == "rmsnorm" else 0
        o.block_mode = 1 if block else 0
        o.vae = 1 if vae else 0
        o.t5 = 1 if t5 else 0
        o.t5_vocab, o.t5_ffn, o.t5_layers = t5_vocab, t5_ffn, t5_layers
        h = C.c_void_p()
        st = Status()
        _raise(self.lib, self.lib.wam_b200_create(C.byref(o), C.byref(h), C.byref(st)), st,
               "wam_b200_create")
        self.h = h
        self.max_batch = max_batch
        g = Geometry()
        self.lib.wam_b200_geometry_of(self.h, C.byref(g))
        self.geometry = {n: getattr(g, n) for n in GEOM_FIELDS}
        self.geometry.update(norm_eps=g.norm_eps, flow_shift=g.flow_shift)
        self._keep = []

    def close(self):
        if getattr(self, "h", None):
            self.lib.wam_b200_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def _requests(self, reqs):
        arr = (Request * len(reqs))()
        keep = []
        for i, r in enumerate(reqs):
            s = _f32(r.state)
            keep.append(s)
            fp = C.POINTER(C.c_float)
            arr[i].state = s.ctypes.data_as(fp)
            arr[i].state_n = s.size
            if r.prompt is not None:
                pr = _f32(r.prompt)
                keep.append(pr)
                arr[i].prompt_emb = pr.ctypes.data_as(fp)
                arr[i].prompt_tokens = (pr.shape[0] if pr.ndim == 2
                                        else pr.size // self.geometry["text_dim"])
            if r.tokens is not None:
                tk = np.ascontiguousarray(r.tokens, np.int32)
                keep.append(tk)
                arr[i].lang_tokens = tk.ctypes.data_as(C.POINTER(C.c_int32))
                arr[i].n_lang = tk.size
                if r.mask is not None:
                    mk = np.ascontiguousarray(r.mask, np.int32)
                    keep.append(mk)
                    arr[i].attention_mask = mk.ctypes.data_as(C.POINTER(C.c_int32))
                    arr[i].attention_mask_n = mk.size
            if r.latent is not None:
                lat = _f32(r.latent)
                keep.append(lat)
                arr[i].ref_latent = lat.ctypes.data_as(fp)
                arr[i].ref_latent_n = lat.size
            if r.images is not None:
                views = [np.ascontiguousarray(v) for v in r.images]
                imgs = (Image * len(views))()
                for j, v in enumerate(views):
                    imgs[j] = Image(v.ctypes.data, int(v.shape[1]), int(v.shape[0]),
                                    0 if v.dtype == np.uint8 else 1)
                keep += views + [imgs]
                arr[i].images = imgs
                arr[i].n_images = len(views)
            if r.noise is not None:
                nz = _f32(r.noise)
                keep.append(nz)
                arr[i].noise = nz.ctypes.data_as(fp)
        return arr, keep

    def _out(self, batch):
        g = self.geometry
        return np.zeros((batch, g["action_chunk"], g["real_action_dim"]), np.float32)

    def predict_batch(self, reqs, stats: bool = False):
        arr, keep = self._requests(reqs)
        out = self._out(len(reqs))
        st, s = Status(), Stats()
        rc = self.lib.wam_b200_predict_batch(self.h, arr, len(reqs),
                                             out.ctypes.data_as(C.POINTER(C.c_float)), out.size,
                                             C.byref(s), C.byref(st))
        _raise(self.lib, rc, st, "wam_b200_predict_batch")
        if stats:
            return out, {f: getattr(s, f) for f, _ in Stats._fields_}
        return out

    def predict(self, req, stats: bool = False):
        r = self.predict_batch([req], stats)
        return (r[0][0], r[1]) if stats else r[0]

    def stage(self, reqs):
        arr, keep = self._requests(reqs)
        self._keep = keep
        st = Status()
        _raise(self.lib, self.lib.wam_b200_stage(self.h, arr, len(reqs), C.byref(st)), st,
               "wam_b200_stage")

    def run(self, batch: int):
        st = Status()
        _raise(self.lib, self.lib.wam_b200_run(self.h, batch, C.byref(st)), st, "wam_b200_run")

    def fetch(self, reqs):
        arr, keep = self._requests(reqs)
        out = self._out(len(reqs))
        st = Status()
        rc = self.lib.wam_b200_fetch(self.h, arr, len(reqs), out.ctypes.data_as(C.POINTER(C.c_float)),
                                     out.size, C.byref(st))
        _raise(self.lib, rc, st, "wam_b200_fetch")
        return out

    def stream(self) -> int:
        return self.lib.wam_b200_stream(self.h) or 0

    def kernel_launches(self, batch: int, with_prompt: bool = True) -> int:
        return self.lib.wam_b200_kernel_launches(self.h, batch, 1 if with_prompt else 0)

    def phase_ms(self) -> dict:
        v = [C.c_float(), C.c_float(), C.c_float()]
        rc = self.lib.wam_b200_phase_ms(self.h, *[C.byref(x) for x in v])
        if rc != 0:
            raise EngineError(rc, "wam_b200_phase_ms")
        return dict(zip(PHASES, (x.value for x in v)))

    def profile(self, batch: int) -> list[dict]:
        """Per-op device times of one chunk on the staged batch (eager, events
        around every op)."""
        n = 20000
        arr = (OpProfile * n)()
        st = Status()
        rc = self.lib.wam_b200_profile(self.h, batch, arr, n, C.byref(st))
        if rc < 0:
            _raise(self.lib, -rc, st, "wam_b200_profile")
        return [{"phase": PHASES[a.phase], "kind": KINDS[a.kind], "launches": a.launches,
                 "ms": a.ms, "bytes": a.bytes, "flops": a.flops, "shape": list(a.shape)}
                for a in arr[:rc]]

    def profile_graph(self, batch: int, phase: str, kind: str, reps: int = 5,
                      lane: int = -1) -> dict:
        """Device time of the (phase, kind) ops of the staged batch replayed
        alone in a CUDA graph (wam_b200_profile_graph_lane; lane -1 = all,
        0 = main stream, 1 = side stream)."""
        out, st = GraphProfile(), Status()
        rc = self.lib.wam_b200_profile_graph_lane(self.h, batch, PHASES.index(phase),
                                                  KINDS.index(kind), lane, reps, C.byref(out),
                                                  C.byref(st))
        _raise(self.lib, rc, st, "wam_b200_profile_graph_lane")
        return {"ms": out.ms, "bytes": out.bytes, "flops": out.flops, "launches": out.launches}

    def block_forward(self, t: float, xv, xa, tv, ta, with_time: bool = False):
        """Config 1: one MoT layer over given hidden states (wam_b200_block_forward).
        xv [V, H], xa [1 + T, E] (state row first), tv [Nt, H], ta [Nt, E] F32.
        Returns (visual out [V, H], action stream out [1 + T, E]) and, with
        with_time, the device time in ms."""
        g = self.geometry
        V, H, E, T = g["grid_h"] * g["grid_w"], g["hidden"], g["action_hidden"], g["action_chunk"]
        arrs = [_f32(a) for a in (xv, xa, tv, ta)]
        fp = C.POINTER(C.c_float)
        inp = BlockInputs(arrs[0].ctypes.data_as(fp), arrs[1].ctypes.data_as(fp),
                          arrs[2].ctypes.data_as(fp), arrs[3].ctypes.data_as(fp), t)
        ov = np.zeros((V, H), np.float32)
        oa = np.zeros((1 + T, E), np.float32)
        ms = C.c_float(0.0)
        st = Status()
        rc = self.lib.wam_b200_block_forward(self.h, C.byref(inp), ov.ctypes.data_as(fp), ov.size,
                                             oa.ctypes.data_as(fp), oa.size, C.byref(ms),
                                             C.byref(st))
        _raise(self.lib, rc, st, "wam_b200_block_forward")
        return (ov, oa, ms.value) if with_time else (ov, oa)

    def reset(self):
        self.lib.wam_b200_reset(self.h)

    def read_tensor(self, name: str, slot: int = 0, layer: int = 0) -> np.ndarray:
        g = self.geometry
        P = 1 + g["grid_h"] * g["grid_w"]
        shapes = {"prefix_k": (g["heads"], P, 128), "prefix_v": (g["heads"], P, 128),
                  "prompt_k": (g["heads"], g["prompt_tokens"], 128),
                  "prompt_v": (g["heads"], g["prompt_tokens"], 128),
                  "velocity": (g["steps"], g["action_chunk"], g["action_dim"])}
        out = np.zeros(shapes[name], np.float32)
        st = Status()
        rc = self.lib.wam_b200_read_tensor(self.h, name.encode(), slot, layer,
                                           out.ctypes.data_as(C.POINTER(C.c_float)), out.size,
                                           C.byref(st))
        _raise(self.lib, rc, st, "wam_b200_read_tensor")
        return out


class Batcher:
    """The batch-capable serving surface over one engine
    (wam_b200_batcher_*): predict() may be called from many threads at once;
    queued requests run together as predict_batch calls of up to the engine's
    max_batch, waiting at most max_wait_us after the first for more."""

    def __init__(self, engine: Engine, max_wait_us: int = 200):
        self.engine = engine
        self.lib = engine.lib
        self.h = C.c_void_p()
        st = Status()
        _raise(self.lib, self.lib.wam_b200_batcher_create(engine.h, max_wait_us, C.byref(self.h),
                                                          C.byref(st)),
               st, "wam_b200_batcher_create")

    def predict(self, req: Req):
        """(action chunk [action_chunk, real_action_dim], batch size it ran in)."""
        arr, keep = self.engine._requests([req])
        out = self.engine._out(1)[0]
        st, s, b = Status(), Stats(), C.c_int()
        rc = self.lib.wam_b200_batcher_predict(self.h, arr, out.ctypes.data_as(C.POINTER(C.c_float)),
                                               out.size, C.byref(s), C.byref(b), C.byref(st))
        _raise(self.lib, rc, st, "wam_b200_batcher_predict")
        return out, b.value

    def counts(self):
        nb, nr = C.c_longlong(), C.c_longlong()
        self.lib.wam_b200_batcher_counts(self.h, C.byref(nb), C.byref(nr))
        return nb.value, nr.value

    def close(self):
        if self.h:
            self.lib.wam_b200_batcher_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
