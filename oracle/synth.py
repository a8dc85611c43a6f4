"""Deterministic synthetic GWP-0.5 weights — TEST INFRASTRUCTURE.

(The geometries and seeded request inputs live in the product package,
wam_b200.workload, and are re-exported here for the tests.)

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

import sys
from pathlib import Path

import numpy as np

_PKG = Path(__file__).resolve().parent.parent / "wam.cpp_b200"
if str(_PKG) not in sys.path:
    sys.path.insert(0, str(_PKG))

from wam_b200.workload import (CONFIG1, CONFIG2, CONFIG2_L1, CONFIG2_L2, PAIR,  # noqa: E402,F401
                               SMALL, TALL, TINY, WIDE, Geometry, Request, make_block_inputs,
                               make_request, statistics)

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


def make_vae_weights(seed: int, z_dim: int = 48) -> dict[str, np.ndarray]:
    """The synthetic Wan VAE encoder weights of csrc/vae.cu (load_weights):
    convolutions N(0, 1 / fan_in), biases N(0, 0.02), RMS gains 1 + N(0, 0.02)."""
    from wam_b200.vision import vae_tensor_specs

    out = {}
    for name, shape in vae_tensor_specs(z_dim):
        n = int(np.prod(shape))
        if name.endswith(".weight"):
            scale, center = 1.0 / float(np.sqrt(float(shape[1] * shape[2] * shape[3]))), 0.0
        elif name.endswith(".bias"):
            scale, center = 0.02, 0.0
        else:
            scale, center = 0.02, 1.0
        out[name] = synth_bits(seed, name, n, scale, center).reshape(shape)
    return out


def make_t5_weights(seed: int, g) -> dict[str, np.ndarray]:
    """The synthetic UMT5 weights of csrc/t5.cu (load_weights): linear maps
    N(0, 1 / fan_in) (q also / sqrt(head_dim)), embedding N(0, 1), relative
    position bias N(0, 0.5), RMS gains 1 + N(0, 0.02)."""
    from wam_b200.text import t5_tensor_specs

    out = {}
    for name, shape in t5_tensor_specs(g):
        n = int(np.prod(shape))
        if name.endswith("norm.weight"):
            scale, center = 0.02, 1.0
        elif name == "t5.token_embd.weight":
            scale, center = 1.0, 0.0
        elif name.endswith(".rel.weight"):
            scale, center = 0.5, 0.0
        else:
            scale, center = 1.0 / float(np.sqrt(float(shape[1]))), 0.0
            if name.endswith(".sa.q.weight"):
                scale /= float(np.sqrt(float(g.head_dim)))
        out[name] = synth_bits(seed, name, n, scale, center).reshape(shape)
    return out
