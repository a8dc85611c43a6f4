"""Q8_0 codec: the restatement used by the device quantiser (q8.cu) checked
bit for bit against the gguf-py package's Q8_0 quantiser / dequantiser (the
reference codec of the GGML format; the wam.cpp reference has no Q8_0 path)."""
import numpy as np
import pytest

gguf = pytest.importorskip("gguf")
from gguf import quants  # noqa: E402


def q8_restated(x):
    """d = max|x| / 127 (F32), q = round-half-away(x * (1/d)), d as fp16."""
    b = x.reshape(-1, 32).astype(np.float32)
    d = np.abs(b).max(axis=1, keepdims=True) / np.float32(127)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    t = (b * inv).astype(np.float32)
    a = np.abs(t)
    fl = np.floor(a)
    r = fl + np.floor(np.float32(2) * (a - fl))
    q = (np.sign(t) * r).astype(np.int8)
    return np.concatenate([d.astype(np.float16).view(np.uint8), q.view(np.uint8)], axis=1)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_q8_restatement_matches_gguf(seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    # ties: values that land exactly on k + 0.5 after scaling, zeros, a zero block
    x[0, :32] = np.linspace(-1, 1, 32, dtype=np.float32) * np.float32(127 / 64)
    x[1, :32] = 0.0
    x[2, 5] = -x[2, :32].max() * 3
    ref = quants.quantize(x, gguf.GGMLQuantizationType.Q8_0).reshape(-1, 34)
    assert np.array_equal(q8_restated(x), ref)
    deq = quants.dequantize(ref.reshape(x.shape[0], -1), gguf.GGMLQuantizationType.Q8_0)
    d = ref[:, :2].copy().view(np.float16).astype(np.float32)
    q = ref[:, 2:].view(np.int8).astype(np.float32)
    assert np.array_equal((q * d).reshape(x.shape), deq)


@pytest.mark.parametrize("seed", [0, 3])
def test_oracle_q8_f32_dequant_matches_gguf(seed):
    """The oracle's config-5 weights are dequantize_row_q8_0's F32 values
    (gguf.quants.dequantize), bit for bit: no BF16 rounding of q * d."""
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(repo)]
    import oracle
    from oracle import synth

    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(64 * 512) * 0.02).astype(np.float32)
    x[:32] = 0.0                                   # zero block: d = 0, q = 0
    x[32:64] = np.float32(1e-6) * np.arange(32)    # tiny block (fp16 d near subnormal)
    x[64:96] = np.linspace(-1, 1, 32, dtype=np.float32) * np.float32(127 / 64)  # ties
    bits = synth.f32_to_bf16_bits(x)
    xf = synth.bf16_bits_to_f32(bits).reshape(-1, 32)
    want = quants.dequantize(quants.quantize(xf, gguf.GGMLQuantizationType.Q8_0),
                             gguf.GGMLQuantizationType.Q8_0).astype(np.float32).reshape(-1)
    got = oracle.q8_roundtrip(bits)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
