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
