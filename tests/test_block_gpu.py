"""one MoT block (layer 0 of the reference's un-cached
forward, run_mot_step, src/models/gwp05/engine/mot.cpp:1008-1067) over given
hidden states, through wam_b200_block_forward, against the oracle's
block_forward (oracle/oracle.cpp) on the same synthetic weights and inputs.

Config 1 as BASELINE states it ("RMSNorm + AdaLN", "SiLU-gated MLP") differs
from the reference (LayerNorm inside AdaLN, GELU(tanh) FFN); both forms are
built and checked. A block's output is its input plus small residual
branches, so the check is on the branches: (out - in) within 5e-2
relative-L2 of the oracle's, for the visual tokens and the action stream, and
the outputs within 1e-2.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED = 20261204


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30))


@pytest.mark.parametrize("geom_name", ["TINY", "CONFIG1"])
@pytest.mark.parametrize("ffn,norm", [("gelu", "layernorm"), ("swiglu", "rmsnorm"),
                                      ("swiglu", "layernorm"), ("gelu", "rmsnorm")])
def test_block_matches_oracle(cuda_device, geom_name, ffn, norm):
    import dataclasses

    import oracle
    from oracle import synth
    from wam_b200.engine import Engine

    geom = dataclasses.replace(getattr(synth, geom_name), layers=1, steps=1)
    if geom_name == "TINY" and ffn == "swiglu":
        geom = dataclasses.replace(geom, ffn=512, action_ffn=512)  # whole 256-row gate / up halves
    x = synth.make_block_inputs(geom, 3)
    eng = Engine(geom, seed=SEED, bias_scale=0.02, prompt_cache=False, ffn=ffn, norm=norm,
                 block=True)
    ov, oa = eng.block_forward(x["t"], x["xv"], x["xa"], x["tv"], x["ta"])
    om = oracle.OracleModel(geom, None, seed=SEED, bias_scale=0.02,
                            ffn_kind=1 if ffn == "swiglu" else 0)
    rv, ra = om.block(x["t"], x["xv"], x["xa"], x["tv"], x["ta"],
                      norm_kind=1 if norm == "rmsnorm" else 0)
    assert np.isfinite(ov).all() and np.isfinite(oa).all()
    xv = x["xv"].astype(np.float32)
    xa = x["xa"].astype(np.float32)
    # inputs enter as BF16 hidden states: compare branches against the BF16 input
    bv = np.asarray(__import__("torch").tensor(xv).bfloat16().float())
    ba = np.asarray(__import__("torch").tensor(xa).bfloat16().float())
    dv, da = rel_l2(ov - bv, rv - bv), rel_l2(oa - ba, ra - ba)
    assert dv < 5e-2, f"visual branch rel-L2 {dv:.3e}"
    assert da < 5e-2, f"action-stream branch rel-L2 {da:.3e}"
    assert rel_l2(ov, rv) < 1e-2 and rel_l2(oa, ra) < 1e-2


def test_block_calls_repeat_and_reject_chunk_calls(cuda_device):
    """Two block calls on new inputs give independent results; a block engine
    refuses predict (it holds one layer and no decoder)."""
    import dataclasses

    from oracle import synth
    from wam_b200.engine import Engine, EngineError, Req

    geom = dataclasses.replace(synth.TINY, layers=1, steps=1)
    eng = Engine(geom, seed=SEED, bias_scale=0.02, prompt_cache=False, block=True)
    x1, x2 = synth.make_block_inputs(geom, 1), synth.make_block_inputs(geom, 2)
    a1 = eng.block_forward(x1["t"], x1["xv"], x1["xa"], x1["tv"], x1["ta"])
    a2 = eng.block_forward(x2["t"], x2["xv"], x2["xa"], x2["tv"], x2["ta"])
    b1 = eng.block_forward(x1["t"], x1["xv"], x1["xa"], x1["tv"], x1["ta"])
    assert np.array_equal(a1[0], b1[0]) and np.array_equal(a1[1], b1[1])
    assert not np.array_equal(a1[1], a2[1])
    r = synth.make_request(geom, 4)
    with pytest.raises(EngineError):
        eng.predict(Req(r.state, r.latent, r.prompt, r.noise))
