"""The UMT5 text encoder on the B200 (csrc/t5.cu: tcgen05 GEMMs, 64-dim
relative-bias attention) against the CPU oracle (oracle/t5.cpp, the reference
run_t5's F32 math with its BF16 rounding points), with the reference's mask
and token checks (validate_prompt_mask, text_encoder.cpp:74-109)."""
import numpy as np
import pytest

from wam_b200.text import T5Geometry, T5_TINY

pytestmark = pytest.mark.gpu

MID = T5Geometry(vocab=3000, hidden=1024, ffn=2816, heads=16, head_dim=64, layers=2,
                 max_tokens=512)


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30))


@pytest.mark.parametrize("g,n", [(T5_TINY, 37), (T5_TINY, 64), (T5_TINY, 1), (MID, 300),
                                 (MID, 512)])
def test_t5_matches_oracle(cuda_device, g, n):
    import oracle
    from oracle import synth
    from wam_b200.text import TextEncoder

    enc = TextEncoder(g, seed=7)
    tok = np.random.default_rng(n).integers(0, g.vocab, n).astype(np.int32)
    out = enc.encode(tok)
    want = oracle.t5_encode(synth.make_t5_weights(7, g), g, tok, g.max_tokens)
    assert out.shape == (g.max_tokens, g.hidden)
    assert np.isfinite(out).all() and (out[n:] == 0).all()
    assert rel_l2(out[:n], want[:n]) < 2e-2, rel_l2(out[:n], want[:n])
    assert np.array_equal(enc.encode(tok), out)  # replay is deterministic
    enc.close()


def test_t5_mask_and_token_checks(cuda_device):
    from wam_b200.text import TextEncoder

    g = T5_TINY
    enc = TextEncoder(g, seed=7)
    tok = np.random.default_rng(3).integers(0, g.vocab, 50).astype(np.int32)
    mask = np.array([1] * 20 + [0] * 30, np.int32)
    a = enc.encode(tok, mask)
    b = enc.encode(tok[:20])
    assert np.array_equal(a, b)
    with pytest.raises(RuntimeError, match="contiguous valid prefix"):
        enc.encode(tok, np.array([1, 0, 1] + [0] * 47, np.int32))
    with pytest.raises(RuntimeError, match="zero or one"):
        enc.encode(tok, np.array([2] * 50, np.int32))
    with pytest.raises(RuntimeError, match="no valid tokens"):
        enc.encode(tok, np.zeros(50, np.int32))
    with pytest.raises(RuntimeError, match="does not match"):
        enc.encode(tok, np.ones(49, np.int32))
    with pytest.raises(RuntimeError, match="outside"):
        enc.encode(np.zeros(g.max_tokens + 1, np.int32))
    bad = tok.copy()
    bad[5] = g.vocab
    with pytest.raises(RuntimeError, match="vocabulary"):
        enc.encode(bad)
    enc.close()
