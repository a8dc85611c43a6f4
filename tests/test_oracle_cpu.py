"""The oracle's own modes, on the CPU: the un-cached mode (the reference's CPU
behaviour, prefix recomputed every step) gives the cached mode's chunk, and the
config-5 mode computes with the exact F32 Q8_0 dequantisation."""
import numpy as np


def test_uncached_mode_equals_cached():
    import oracle
    from oracle import synth

    g = synth.TINY
    r = synth.make_request(g, 3)
    a = oracle.OracleModel(g, None, seed=5, bias_scale=0.02).predict(r)["action"]
    b = oracle.OracleModel(g, None, seed=5, bias_scale=0.02).set_uncached().predict(r)["action"]
    assert np.array_equal(a, b)


def test_q8_mode_uses_f32_dequantised_weights():
    """The Q8_0 mode changes the chunk (its weights are the round-tripped
    ones; their F32 values are pinned to gguf-py in test_q8_cpu.py) and stays
    close to the BF16 model's."""
    import oracle
    from oracle import synth

    g = synth.TINY
    r = synth.make_request(g, 4)
    q8 = oracle.OracleModel(g, None, seed=6, bias_scale=0.02).quantize_q8().predict(r)["action"]
    bf = oracle.OracleModel(g, None, seed=6, bias_scale=0.02).predict(r)["action"]
    assert np.isfinite(q8).all()
    assert not np.array_equal(q8, bf)
    rel = np.linalg.norm(q8 - bf) / np.linalg.norm(bf)
    assert rel < 5e-2
