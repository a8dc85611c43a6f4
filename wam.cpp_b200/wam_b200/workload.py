"""BASELINE workloads of the GWP-0.5 MoT engine: model geometries and seeded
synthetic requests.

The geometry mirrors the reference artifact's gwp05.* keys
(src/models/gwp05/artifact.cpp:20-94; C struct wam_b200_geometry). CONFIG2 is
BASELINE config 2 (the full GWP-0.5-shaped MoT); the smaller presets are the
parity-test geometries. make_request() draws a request's inputs (state, VAE
latent, prompt embedding, initial noise) from N(0, 1) with numpy's PCG64 keyed
by the request seed: the synthetic stand-in for camera latents and T5 prompt
embeddings, which do not exist in this tree.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass
class Geometry:
    hidden: int = 3072
    layers: int = 30
    heads: int = 24
    ffn: int = 14336
    action_hidden: int = 3072
    action_ffn: int = 14336
    action_dim: int = 32
    real_state_dim: int = 14
    real_action_dim: int = 14
    num_embodiments: int = 1
    embodiment_id: int = 0
    grid_h: int = 32
    grid_w: int = 24
    vae_z: int = 48
    action_chunk: int = 48
    steps: int = 10
    prompt_tokens: int = 512
    text_dim: int = 4096
    norm_eps: float = 1e-6
    flow_shift: float = 1.0

    @property
    def visual_tokens(self) -> int:
        return self.grid_h * self.grid_w

    @property
    def prefix_tokens(self) -> int:
        return 1 + self.visual_tokens


# BASELINE config 2 (full GWP-0.5-shaped MoT) and small parity configs.
CONFIG2 = Geometry()
TINY = Geometry(hidden=256, layers=2, heads=2, ffn=512, action_hidden=256, action_ffn=384,
                grid_h=4, grid_w=4, vae_z=16, action_chunk=16, steps=3, prompt_tokens=16,
                text_dim=128)
SMALL = Geometry(hidden=512, layers=3, heads=4, ffn=1024, action_hidden=384, action_ffn=768,
                 grid_h=6, grid_w=8, vae_z=48, action_chunk=48, steps=4, prompt_tokens=64,
                 text_dim=256)
# Config-2 widths (H = E = 3072, F = 14336, 24 heads, 32 x 24 visual grid, 512 x
# 4096 prompt, 48 x 32 actions) with fewer layers and steps: the parity-test
# and smoke geometries of the benched configuration (same kernels, split-K
# plans, persistent GEMMs and attention splits as the full model).
CONFIG2_L2 = Geometry(layers=2, steps=2)
# one MoT block at config-2 widths (768 visual tokens, 512
# text tokens as cross-attention keys, 48 action tokens + the state token).
CONFIG1 = Geometry(layers=1, steps=1)
CONFIG2_L1 = Geometry(layers=1, steps=2)
# 144 visual tokens: the prefix attention (145 / 144 queries) runs as 128-query
# tensor-core tiles.
TALL = Geometry(hidden=256, layers=2, heads=2, ffn=512, action_hidden=256, action_ffn=384,
                grid_h=12, grid_w=12, vae_z=16, action_chunk=16, steps=2, prompt_tokens=16,
                text_dim=128)
# 320 visual and 272 prompt tokens: the prefix and prompt GEMMs (>= 256 token
# rows) run on CTA pairs, split over 2 or 4 pairs where their tiles are few.
PAIR = Geometry(hidden=512, layers=2, heads=4, ffn=1024, action_hidden=512, action_ffn=1024,
                grid_h=16, grid_w=20, vae_z=16, action_chunk=16, steps=2, prompt_tokens=272,
                text_dim=256)
WIDE = Geometry(hidden=1536, layers=2, heads=12, ffn=3072, action_hidden=1536, action_ffn=3072,
                grid_h=4, grid_w=4, vae_z=16, action_chunk=48, steps=2, prompt_tokens=32,
                text_dim=256)


def statistics(g: Geometry) -> dict[str, np.ndarray]:
    """state/action q01/q99 statistics (F32 [action_dim]) of the synthetic artifact."""
    i = np.arange(g.action_dim, dtype=np.float32)
    lo = (-1.0 - 0.01 * i).astype(np.float32)
    hi = (1.0 + 0.02 * i).astype(np.float32)
    return {"state_q01": lo, "state_q99": hi, "action_q01": lo.copy(), "action_q99": hi.copy()}


@dataclass
class Request:
    state: np.ndarray   # [real_state_dim]
    latent: np.ndarray  # [vae_z, 2 gh, 2 gw]
    prompt: np.ndarray  # [prompt_tokens, text_dim]
    noise: np.ndarray   # [T, A]
    extra: dict = field(default_factory=dict)


def make_block_inputs(g: Geometry, seed: int) -> dict:
    """Config-1 inputs, N(0, 1) F32: visual [V, H], action stream [1 + T, E]
    (state token first), the experts' text hidden states [Nt, H] / [Nt, E]
    (one draw used for both when E == H), and a timestep in [0, 1000)."""
    r = np.random.Generator(np.random.PCG64(seed))
    xv = r.standard_normal((g.visual_tokens, g.hidden), dtype=np.float32)
    xa = r.standard_normal((1 + g.action_chunk, g.action_hidden), dtype=np.float32)
    tv = r.standard_normal((g.prompt_tokens, g.hidden), dtype=np.float32)
    ta = tv.copy() if g.action_hidden == g.hidden else r.standard_normal(
        (g.prompt_tokens, g.action_hidden), dtype=np.float32)
    t = float(r.uniform(0.0, 1000.0))
    return {"xv": xv, "xa": xa, "tv": tv, "ta": ta, "t": t}


def make_request(g: Geometry, seed: int) -> Request:
    r = np.random.Generator(np.random.PCG64(seed))
    return Request(
        state=r.standard_normal(g.real_state_dim, dtype=np.float32),
        latent=r.standard_normal((g.vae_z, 2 * g.grid_h, 2 * g.grid_w), dtype=np.float32),
        prompt=r.standard_normal((g.prompt_tokens, g.text_dim), dtype=np.float32),
        noise=r.standard_normal((g.action_chunk, g.action_dim), dtype=np.float32),
    )


# Camera views of the vision front-end: three 640 x 480 RGB frames (the
# LeRobot camera size) onto config 2's 768 x 1024 canvas (image_width =
# grid_w * 32, image_height = grid_h * 32).
VIEWS_CONFIG2 = ((480, 640), (480, 640), (480, 640))


def make_views(seed: int, sizes=VIEWS_CONFIG2, formats=("u8", "u8", "u8")) -> list[np.ndarray]:
    """Seeded synthetic camera views, HWC RGB: uint8 uniform over 0..255
    ("u8") or float32 uniform in [0, 1) ("f32"), one PCG64 stream per view."""
    out = []
    for i, ((h, w), f) in enumerate(zip(sizes, formats)):
        rng = np.random.Generator(np.random.PCG64([seed, i]))
        if f == "u8":
            out.append(rng.integers(0, 256, (h, w, 3), dtype=np.uint8))
        elif f == "f32":
            out.append(rng.random((h, w, 3), dtype=np.float32))
        else:
            raise ValueError(f)
    return out
