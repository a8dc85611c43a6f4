"""End-to-end parity of the CUDA engine against the CPU oracle (oracle/).

Both sides use the same synthetic BF16 weights (bit-identical generator, see
test_ops_gpu.py::test_synthetic_weights_bit_exact) and the same seeded inputs.
Tolerances: per-layer K/V caches within 2e-2
relative-L2, velocities and final action chunks within 5e-2 relative-L2.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED = 20261201


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30))


def _setup(geom, bias_scale=0.02, max_batch=1, graphs=True):
    import oracle
    from oracle import synth
    from wam_b200.engine import Engine

    w = synth.make_weights(geom, SEED, bias_scale=bias_scale)
    om = oracle.OracleModel(geom, w)
    eng = Engine(geom, seed=SEED, bias_scale=bias_scale, max_batch=max_batch, graphs=graphs,
                 prompt_cache=False)
    return om, eng


def _req(geom, seed):
    from oracle import synth
    from wam_b200.engine import Req

    r = synth.make_request(geom, seed)
    return r, Req(r.state, r.latent, r.prompt, r.noise)


@pytest.mark.parametrize("geom_name", ["TINY", "SMALL", "TALL", "PAIR"])
def test_engine_matches_oracle(cuda_device, geom_name):
    from oracle import synth

    geom = getattr(synth, geom_name)
    om, eng = _setup(geom)
    r, er = _req(geom, 11)
    ref = om.predict(r, dumps=True)
    out = eng.predict(er)
    for layer in range(geom.layers):
        for name in ("prefix_k", "prefix_v", "prompt_k", "prompt_v"):
            got = eng.read_tensor(name, 0, layer)
            err = rel_l2(got, ref[name][layer])
            assert err < 2e-2, f"{name} layer {layer}: rel-L2 {err:.3e}"
    vel = eng.read_tensor("velocity")
    for s in range(geom.steps):
        err = rel_l2(vel[s], ref["velocity"][s])
        assert err < 5e-2, f"velocity step {s}: rel-L2 {err:.3e}"
    assert np.isfinite(out).all()
    assert rel_l2(out, ref["action"]) < 5e-2


@pytest.mark.parametrize("geom_name", ["TINY", "SMALL"])
def test_engine_q8_matches_oracle(cuda_device, geom_name):
    """Config-5 policy: Q8_0 linear weights (quantised on the device, gguf-py
    rules); the oracle runs on the gguf-py dequantised weights."""
    pytest.importorskip("gguf")
    import oracle
    from oracle import synth
    from wam_b200.engine import Engine

    geom = getattr(synth, geom_name)
    w = synth.quantize_q8_linear(geom, synth.make_weights(geom, SEED, bias_scale=0.02))
    om = oracle.OracleModel(geom, w)
    eng = Engine(geom, seed=SEED, bias_scale=0.02, prompt_cache=False, weights="q8_0")
    r, er = _req(geom, 13)
    ref = om.predict(r, dumps=True)
    out = eng.predict(er)
    for layer in range(geom.layers):
        for name in ("prefix_k", "prefix_v", "prompt_k", "prompt_v"):
            err = rel_l2(eng.read_tensor(name, 0, layer), ref[name][layer])
            assert err < 2e-2, f"{name} layer {layer}: rel-L2 {err:.3e}"
    vel = eng.read_tensor("velocity")
    for s in range(geom.steps):
        assert rel_l2(vel[s], ref["velocity"][s]) < 5e-2
    assert np.isfinite(out).all()
    assert rel_l2(out, ref["action"]) < 5e-2


def test_graph_and_eager_identical(cuda_device):
    from oracle import synth
    from wam_b200.engine import Engine

    geom = synth.TINY
    r, er = _req(geom, 5)
    a = Engine(geom, seed=SEED, bias_scale=0.02, graphs=True).predict(er)
    b = Engine(geom, seed=SEED, bias_scale=0.02, graphs=False).predict(er)
    assert np.array_equal(a, b)


def test_batch_equals_single_requests(cuda_device):
    from oracle import synth
    from wam_b200.engine import Engine

    geom = synth.TINY
    eng = Engine(geom, seed=SEED, bias_scale=0.02, max_batch=3, prompt_cache=False)
    reqs = [_req(geom, 100 + i)[1] for i in range(3)]
    batched = eng.predict_batch(reqs)
    for i, rq in enumerate(reqs):
        single = eng.predict_batch([rq])[0]
        assert rel_l2(single, batched[i]) < 1e-2


def test_prompt_cache_hit_is_identical(cuda_device):
    from oracle import synth
    from wam_b200.engine import Engine

    geom = synth.TINY
    eng = Engine(geom, seed=SEED, bias_scale=0.02, prompt_cache=True)
    _, rq = _req(geom, 9)
    a, sa = eng.predict(rq, stats=True)
    b, sb = eng.predict(rq, stats=True)
    assert sa["prompt_cache_hit"] == 0 and sb["prompt_cache_hit"] == 1
    assert np.array_equal(a, b)
    eng.reset()
    c, sc = eng.predict(rq, stats=True)
    assert sc["prompt_cache_hit"] == 0 and np.array_equal(a, c)


def test_invalid_inputs_fail_loudly(cuda_device):
    from oracle import synth
    from wam_b200.engine import Engine, EngineError, Req

    geom = synth.TINY
    eng = Engine(geom, seed=SEED)
    r, rq = _req(geom, 3)
    bad = r.state.copy()
    bad[0] = np.nan
    with pytest.raises(EngineError, match="NaN"):
        eng.predict(Req(bad, r.latent, r.prompt, r.noise))
    with pytest.raises(EngineError, match="latent"):
        eng.predict(Req(r.state, r.latent[:1], r.prompt, r.noise))
    # the engine stays usable after rejected requests
    assert np.isfinite(eng.predict(rq)).all()


def test_engine_pair_gemm_matches_oracle(cuda_device):
    """The engine with WAM_B200_GEMM_PAIR=1 (every GEMM of >= 256 token rows on
    CTA pairs: the PAIR geometry's prefix and prompt GEMMs, split over pairs
    through the engine's workspace) against the oracle. The switch is read when
    the library loads, so this runs in a child process."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parents[1]
    code = (
        "import sys; sys.path[:0] = [%r, %r]\n"
        "import numpy as np\n"
        "from tests.test_engine_gpu import _setup, _req, rel_l2\n"
        "from oracle import synth\n"
        "geom = synth.PAIR\n"
        "om, eng = _setup(geom)\n"
        "r, er = _req(geom, 13)\n"
        "ref = om.predict(r, dumps=True)\n"
        "out = eng.predict(er)\n"
        "errs = [rel_l2(eng.read_tensor(n, 0, l), ref[n][l]) for l in range(geom.layers)\n"
        "        for n in ('prefix_k', 'prefix_v', 'prompt_k', 'prompt_v')]\n"
        "vel = eng.read_tensor('velocity')\n"
        "verr = [rel_l2(vel[s], ref['velocity'][s]) for s in range(geom.steps)]\n"
        "aerr = rel_l2(out, ref['action'])\n"
        "print('kv', max(errs), 'vel', max(verr), 'action', aerr)\n"
        "assert max(errs) < 2e-2 and max(verr) < 5e-2 and aerr < 5e-2 and np.isfinite(out).all()\n"
    ) % (str(repo), str(repo / "wam.cpp_b200"))
    env = dict(os.environ, WAM_B200_GEMM_PAIR="1")
    res = subprocess.run([sys.executable, "-c", code], env=env, cwd=str(repo),
                         capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]


def test_profile_graph_lanes(cuda_device):
    """wam_b200_profile_graph_lane: the prefix GEMMs of the main lane (visual
    tokens) and of the side lane (state token) add up to all of them, in
    launches, FLOPs and bytes; each replay is timed."""
    from oracle import synth
    from wam_b200.engine import Engine

    geom = synth.TINY
    eng = Engine(geom, seed=SEED, bias_scale=0.02, prompt_cache=False)
    _, rq = _req(geom, 5)
    eng.stage([rq])
    eng.run(1)
    both = eng.profile_graph(1, "prefix", "gemm", reps=2)
    main = eng.profile_graph(1, "prefix", "gemm", reps=2, lane=0)
    side = eng.profile_graph(1, "prefix", "gemm", reps=2, lane=1)
    assert main["launches"] > 0 and side["launches"] > 0
    assert main["launches"] + side["launches"] == both["launches"]
    assert abs(main["flops"] + side["flops"] - both["flops"]) <= 1e-6 * both["flops"]
    assert abs(main["bytes"] + side["bytes"] - both["bytes"]) <= 1e-6 * both["bytes"]
    assert main["ms"] > 0 and side["ms"] > 0 and both["ms"] > 0
    with pytest.raises(RuntimeError):
        eng.profile_graph(1, "prefix", "gemm", reps=1, lane=2)
