"""Deterministic synthetic GWP-0.5 weights and inputs — TEST INFRASTRUCTURE.

The same integer-hash generator runs on the device inside the engine
(launch_synth_bf16 in wam.cpp_b200/csrc/elementwise.cu): every BF16 value is a
function of (seed, tensor name, element index) computed with integer ops and
two correctly rounded F32 operations, so host and device produce identical bits.

  tensor_seed = splitmix64(seed ^ fnv1a64(name))
  h_i         = mix64(tensor_seed + (i + 1) * 0x9E3779B97F4A7C15)
  z_i         = (u0 + u1 + u2 + u3 - 131070) with u_j the four 16-bit lanes of h_i
  w_i         = bf16(f32(z_i) * f32(scale / 37837.2269...) + f32(center))

z is an Irwin-Hall(4) approximation of N(0, 1) scaled to unit variance.
Tensor names and shapes follow the reference's compact GGUF naming
(src/models/gwp05/engine/weights.cpp:116-167, artifact.cpp:96-118).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)
IRWIN_HALL4_STD = float(np.sqrt(4.0 * (65536.0 ** 2 - 1.0) / 12.0))


def fnv1a64(name: str) -> int:
    h = 0xCBF29CE484222325
    for b in name.encode():
        h ^= b
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def _mix(z):
    z = np.asarray(z, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * M1
        z = (z ^ (z >> np.uint64(27))) * M2
    return z ^ (z >> np.uint64(31))


def splitmix64(x: int) -> int:
    with np.errstate(over="ignore"):
        return int(_mix(np.uint64(x) + GOLDEN))


def tensor_seed(seed: int, name: str) -> int:
    return splitmix64((seed ^ fnv1a64(name)) & 0xFFFFFFFFFFFFFFFF)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    return u.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def synth_bits(seed: int, name: str, n: int, scale: float, center: float) -> np.ndarray:
    """BF16 bit patterns of the synthetic tensor `name` with n elements."""
    ts = np.uint64(tensor_seed(seed, name))
    out = np.empty(n, dtype=np.uint16)
    k = np.float32(scale / IRWIN_HALL4_STD)
    c = np.float32(center)
    chunk = 1 << 22
    for s in range(0, n, chunk):
        idx = np.arange(s + 1, min(n, s + chunk) + 1, dtype=np.uint64)
        with np.errstate(over="ignore"):
            h = _mix(ts + idx * GOLDEN)
        mask = np.uint64(0xFFFF)
        z = ((h & mask) + ((h >> np.uint64(16)) & mask) + ((h >> np.uint64(32)) & mask)
             + (h >> np.uint64(48))).astype(np.int64) - 131070
        v = z.astype(np.float32) * k + c
        out[s:s + len(idx)] = f32_to_bf16_bits(v)
    return out


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
# Action-expert widths that are multiples of 256 with the config-2 chunk of 48
# tokens: the engine runs these denoise steps as its persistent step kernel.
STEPK = Geometry(hidden=512, layers=3, heads=4, ffn=1024, action_hidden=512, action_ffn=1024,
                 grid_h=4, grid_w=6, vae_z=16, action_chunk=48, steps=3, prompt_tokens=32,
                 text_dim=256)
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


def tensor_specs(g: Geometry) -> list[tuple[str, tuple[int, ...]]]:
    """(compact name, numpy shape) of every BF16 tensor the MoT path reads.
    Shapes are row-major numpy shapes, i.e. reversed GGUF ne."""
    E, H, A, D = g.action_hidden, g.hidden, g.action_dim, g.text_dim
    emb = g.num_embodiments
    s: list[tuple[str, tuple[int, ...]]] = [
        ("gwp.patch.weight", (H, g.vae_z, 2, 2)), ("gwp.patch.bias", (H,)),
    ]
    for comp in ("state", "action"):
        s += [(f"gwp.{comp}.in.weight", (emb, A, 128)), (f"gwp.{comp}.in.bias", (emb, 128)),
              (f"gwp.{comp}.mid.weight", (128, 128)), (f"gwp.{comp}.mid.bias", (128,)),
              (f"gwp.{comp}.out.weight", (E, 128)), (f"gwp.{comp}.out.bias", (E,))]
    s += [("gwp.decode.in.weight", (128, E)), ("gwp.decode.in.bias", (128,)),
          ("gwp.decode.mid.weight", (128, 128)), ("gwp.decode.mid.bias", (128,)),
          ("gwp.decode.out.weight", (emb, 128, A)), ("gwp.decode.out.bias", (emb, A)),
          ("gwp.action_mod", (1, 2, E))]
    for comp, W in (("acond", E), ("cond", H)):
        s += [(f"gwp.{comp}.time.0.weight", (W, 256)), (f"gwp.{comp}.time.0.bias", (W,)),
              (f"gwp.{comp}.time.1.weight", (W, W)), (f"gwp.{comp}.time.1.bias", (W,)),
              (f"gwp.{comp}.time.out.weight", (6 * W, W)), (f"gwp.{comp}.time.out.bias", (6 * W,)),
              (f"gwp.{comp}.text.0.weight", (W, D)), (f"gwp.{comp}.text.0.bias", (W,)),
              (f"gwp.{comp}.text.1.weight", (W, W)), (f"gwp.{comp}.text.1.bias", (W,))]
    for layer in range(g.layers):
        for x, W, F in (("a", E, g.action_ffn), ("v", H, g.ffn)):
            p = f"gwp.blk.{layer}.{x}"
            s += [(f"{p}.sa.qkv.weight", (3 * H, W)), (f"{p}.sa.qkv.bias", (3 * H,)),
                  (f"{p}.sa.qn.weight", (H,)), (f"{p}.sa.kn.weight", (H,)),
                  (f"{p}.sa.o.weight", (W, H)), (f"{p}.sa.o.bias", (W,)),
                  (f"{p}.ca.q.weight", (H, W)), (f"{p}.ca.q.bias", (H,)),
                  (f"{p}.ca.k.weight", (H, W)), (f"{p}.ca.k.bias", (H,)),
                  (f"{p}.ca.vproj.weight", (H, W)), (f"{p}.ca.vproj.bias", (H,)),
                  (f"{p}.ca.o.weight", (W, H)), (f"{p}.ca.o.bias", (W,)),
                  (f"{p}.ca.qn.weight", (H,)), (f"{p}.ca.kn.weight", (H,)),
                  (f"{p}.ca_norm.weight", (W,)), (f"{p}.ca_norm.bias", (W,)),
                  (f"{p}.ffn.in.weight", (F, W)), (f"{p}.ffn.in.bias", (F,)),
                  (f"{p}.ffn.out.weight", (W, F)), (f"{p}.ffn.out.bias", (W,)),
                  (f"{p}.mod", (1, 6, W))]
    return s


def init_rule(name: str, bias_scale: float) -> tuple[float, float]:
    """(scale, center) of a tensor's synthetic distribution. Mirrors
    synth_rule() in wam.cpp_b200/csrc/weights.cpp."""
    if name.endswith(".bias"):
        return bias_scale, 0.0
    if name.endswith((".qn.weight", ".kn.weight", ".ca_norm.weight")):
        return 0.02, 1.0
    return 0.02, 0.0


def make_weights(g: Geometry, seed: int, bias_scale: float = 0.02) -> dict[str, np.ndarray]:
    out = {}
    for name, shape in tensor_specs(g):
        scale, center = init_rule(name, bias_scale)
        out[name] = synth_bits(seed, name, int(np.prod(shape)), scale, center).reshape(shape)
    return out


def linear_inner(name: str, g: Geometry) -> int:
    """Row length of a linear layer's weight as the engine's Q8_0 policy sees it
    (0: not a linear weight). Mirrors linear_inner() in wam.cpp_b200/csrc/engine.cu."""
    if not name.endswith(".weight") or name.endswith((".qn.weight", ".kn.weight",
                                                        "ca_norm.weight")):
        return 0
    E, H = g.action_hidden, g.hidden
    if name == "gwp.patch.weight":
        return g.vae_z * 4
    if name.endswith(".in.weight") and name.startswith(("gwp.state", "gwp.action")):
        return 128
    if name.endswith(".mid.weight") or name in ("gwp.state.out.weight", "gwp.action.out.weight"):
        return 128
    if name == "gwp.decode.in.weight":
        return E
    if name == "gwp.decode.out.weight":
        return g.action_dim
    if name.endswith(".time.0.weight"):
        return 256
    if name.endswith(".text.0.weight"):
        return g.text_dim
    if name.startswith("gwp.acond"):
        return E
    if name.startswith("gwp.cond"):
        return H
    act = ".a." in name
    W, F = (E, g.action_ffn) if act else (H, g.ffn)
    if name.endswith((".sa.o.weight", ".ca.o.weight")):
        return H
    if name.endswith(".ffn.out.weight"):
        return F
    return W


def quantize_q8_linear(g: Geometry, weights: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    """Config-5 weights: every linear weight whose rows are whole 32-value
    blocks goes through the gguf-py Q8_0 codec (quantise, dequantise) and back
    to BF16, the values the engine's Q8_0 GEMM computes with."""
    import gguf
    from gguf import quants

    out = dict(weights)
    for name, w in weights.items():
        inner = linear_inner(name, g)
        if inner <= 0 or inner % 32:
            continue
        f = bf16_bits_to_f32(w.reshape(-1)).reshape(-1, 32)
        q = quants.quantize(f, gguf.GGMLQuantizationType.Q8_0)
        d = quants.dequantize(q, gguf.GGMLQuantizationType.Q8_0).astype(np.float32)
        out[name] = f32_to_bf16_bits(d.reshape(-1)).reshape(w.shape)
    return out


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


def make_request(g: Geometry, seed: int) -> Request:
    r = np.random.Generator(np.random.PCG64(seed))
    return Request(
        state=r.standard_normal(g.real_state_dim, dtype=np.float32),
        latent=r.standard_normal((g.vae_z, 2 * g.grid_h, 2 * g.grid_w), dtype=np.float32),
        prompt=r.standard_normal((g.prompt_tokens, g.text_dim), dtype=np.float32),
        noise=r.standard_normal((g.action_chunk, g.action_dim), dtype=np.float32),
    )
