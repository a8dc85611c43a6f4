"""UMT5 host pieces on the CPU, pinned to the reference's own compiled
functions (tests/golden/make_golden_text.py): the relative position buckets of
the C ABI and of the oracle, and the oracle's timestep embedding."""
import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_text.json"


def test_relative_bucket_matches_reference():
    from wam_b200.text import relative_bucket

    g = json.loads(GOLDEN.read_text())
    got = [relative_bucket(r, 32, 128) for r in g["relative"]]
    assert got == g["bucket_32_128"]


def test_oracle_timestep_embedding_matches_reference():
    import oracle

    g = json.loads(GOLDEN.read_text())
    for case in g["timestep_embedding"]:
        want = np.array(case["bits"], np.uint32).view(np.float32)
        got = oracle.timestep_embedding(case["t"], case["dim"])
        # The oracle restates the formula with the same float operations.
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), case["t"]


def test_t5_tensor_specs_count():
    from wam_b200.text import T5_XXL, t5_tensor_specs

    # gwp05_gguf.py component_expected_counts: t5 = 2 + 10 * t5_layers.
    assert len(t5_tensor_specs(T5_XXL)) == 2 + 10 * T5_XXL.layers


def test_oracle_t5_runs_and_pads():
    import oracle
    from oracle import synth
    from wam_b200.text import T5_TINY

    w = synth.make_t5_weights(5, T5_TINY)
    tok = np.random.default_rng(1).integers(0, T5_TINY.vocab, 37)
    out = oracle.t5_encode(w, T5_TINY, tok, T5_TINY.max_tokens)
    assert np.isfinite(out).all() and (out[37:] == 0).all() and out[:37].std() > 0.1
