"""CPU tests: the C ABI loads and exports what it declares, the engine's and the
oracle's host arithmetic match golden vectors produced by the reference's own
scheduler.cpp / semantics.cpp (tests/golden/make_golden.py), and the oracle
itself behaves (determinism, sensitivity, shapes). No GPU, no compute calls
into the CUDA library.
"""
import ctypes as C
import json
import re
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
GOLDEN = json.loads((REPO / "tests" / "golden" / "reference_host.json").read_text())
f32p = C.POINTER(C.c_float)


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def from_bits(b):
    return np.asarray(b, np.uint32).view(np.float32)


@pytest.fixture(scope="module")
def lib():
    import wam_b200

    return wam_b200.load()


def test_abi_exports_every_declared_symbol(lib):
    header = (REPO / "include" / "wam_b200.h").read_text()
    names = re.findall(r"WAM_B200_API\s+[\w\s\*]+?\b(wam_b200_\w+)\s*\(", header)
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/wam_b200.h but not exported"
    assert lib.wam_b200_abi_version() == 2


def test_engine_schedule_matches_reference(lib):
    for case in GOLDEN["schedules"]:
        n = case["steps"]
        ts = np.zeros(n, np.float32)
        sg = np.zeros(n + 1, np.float32)
        assert lib.wam_b200_flow_schedule(n, case["shift"], ts.ctypes.data_as(f32p),
                                          sg.ctypes.data_as(f32p)) == 0
        assert bits(ts).tolist() == case["timesteps_bits"]
        assert bits(sg).tolist() == case["sigmas_bits"]


def test_oracle_schedule_matches_reference():
    import oracle

    for case in GOLDEN["schedules"]:
        ts, sg = oracle.schedule(case["steps"], case["shift"])
        assert bits(ts).tolist() == case["timesteps_bits"]
        assert bits(sg).tolist() == case["sigmas_bits"]


def test_visual_positions_match_reference(lib):
    import oracle

    for case in GOLDEN["visual_positions"]:
        gh, gw = case["grid"]
        thw = np.zeros(gh * gw * 3, np.int32)
        assert lib.wam_b200_visual_positions(gh, gw, thw.ctypes.data_as(C.POINTER(C.c_int))) == 0
        thw = thw.reshape(-1, 3)
        assert thw[:, 0].tolist() == case["t"]
        assert thw[:, 1].tolist() == case["h"]
        assert thw[:, 2].tolist() == case["w"]
        t, h, w = (np.zeros(gh * gw, np.int32) for _ in range(3))
        i32p = C.POINTER(C.c_int32)
        oracle.lib().oracle_visual_positions(gh, gw, t.ctypes.data_as(i32p), h.ctypes.data_as(i32p),
                                             w.ctypes.data_as(i32p))
        assert (t.tolist(), h.tolist(), w.tolist()) == (case["t"], case["h"], case["w"])


def test_action_positions_match_reference():
    # The engine applies action RoPE at positions pos_base + row with pos_base = 1
    # on the cached path (no state token) and 0 for the prefix state token.
    for case in GOLDEN["action_positions"]:
        base = 0 if case["include_state"] else 1
        n = case["tokens"] + case["include_state"]
        assert case["positions"] == list(range(base, base + n))


def test_state_normalisation_matches_reference(lib):
    for case in GOLDEN["normalize_state"]:
        s = np.asarray(case["state"], np.float32)
        q01 = np.asarray(case["q01"], np.float32)
        q99 = np.asarray(case["q99"], np.float32)
        out = np.zeros(32, np.float32)
        assert lib.wam_b200_normalize_state(s.ctypes.data_as(f32p), s.size, 32,
                                            q01.ctypes.data_as(f32p), q99.ctypes.data_as(f32p),
                                            out.ctypes.data_as(f32p)) == 0
        assert bits(out).tolist() == case["out_bits"]


def test_state_normalisation_rejects_nan(lib):
    s = np.array([0.1, np.nan], np.float32)
    q = np.zeros(4, np.float32)
    out = np.zeros(4, np.float32)
    assert lib.wam_b200_normalize_state(s.ctypes.data_as(f32p), 2, 4, q.ctypes.data_as(f32p),
                                        q.ctypes.data_as(f32p), out.ctypes.data_as(f32p)) != 0


def test_postprocess_matches_reference(lib):
    for case in GOLDEN["postprocess"]:
        a = np.asarray(case["action"], np.float32)
        st = np.asarray(case["state"], np.float32)
        q01 = np.asarray(case["q01"], np.float32)
        q99 = np.asarray(case["q99"], np.float32)
        out = np.zeros(case["steps"] * case["real"], np.float32)
        assert lib.wam_b200_postprocess_action(a.ctypes.data_as(f32p), case["steps"], 32,
                                               case["real"], q01.ctypes.data_as(f32p),
                                               q99.ctypes.data_as(f32p), st.ctypes.data_as(f32p),
                                               out.ctypes.data_as(f32p)) == 0
        assert bits(out).tolist() == case["out_bits"]


def test_synthetic_generator_known_answer():
    """Pins the synthetic-weight generator (shared by the engine's device kernel)."""
    from oracle import synth

    v = synth.synth_bits(1234, "gwp.blk.0.a.sa.qkv.weight", 8, 0.02, 0.0)
    w = synth.bf16_bits_to_f32(v)
    assert np.all(np.abs(w) < 0.02 * 3.5)
    again = synth.synth_bits(1234, "gwp.blk.0.a.sa.qkv.weight", 8, 0.02, 0.0)
    assert np.array_equal(v, again)
    big = synth.bf16_bits_to_f32(synth.synth_bits(7, "x", 1 << 18, 1.0, 0.0))
    assert abs(float(big.mean())) < 0.01 and abs(float(big.std()) - 1.0) < 0.01


def test_engine_tensor_seed_matches_generator(lib):
    from oracle import synth

    for name in ("gwp.patch.weight", "gwp.blk.12.v.ffn.out.weight"):
        assert lib.wam_b200_tensor_seed(99, name.encode()) == synth.tensor_seed(99, name)


@pytest.fixture(scope="module")
def tiny_oracle():
    import oracle
    from oracle import synth

    g = synth.TINY
    return g, oracle.OracleModel(g, synth.make_weights(g, 42, bias_scale=0.02)), synth


def test_oracle_deterministic_and_finite(tiny_oracle):
    g, om, synth = tiny_oracle
    r = synth.make_request(g, 1)
    a = om.predict(r, dumps=True)
    b = om.predict(r, dumps=True)
    assert np.array_equal(a["action"], b["action"])
    for k, v in a.items():
        assert np.isfinite(v).all(), k
    assert a["prefix_k"].shape == (g.layers, g.heads, g.prefix_tokens, 128)
    assert a["velocity"].shape == (g.steps, g.action_chunk, g.action_dim)


def test_oracle_is_sensitive_to_every_layer(tiny_oracle):
    """A planted change to the last layer's action weights moves the velocity:
    the oracle does not silently skip layers."""
    import oracle

    g, om, synth = tiny_oracle
    w = synth.make_weights(g, 42, bias_scale=0.02)
    name = f"gwp.blk.{g.layers - 1}.a.ffn.out.weight"
    w[name] = (w[name].astype(np.int32) ^ 0x0040).astype(np.uint16)
    planted = oracle.OracleModel(g, w)
    r = synth.make_request(g, 1)
    base = om.predict(r, dumps=True)["velocity"]
    moved = planted.predict(r, dumps=True)["velocity"]
    assert not np.array_equal(base, moved)


def test_oracle_prompt_padding_is_zero_rows(tiny_oracle):
    """Prompts shorter than prompt_tokens are zero-padded (pad_prompt_embedding,
    semantics.cpp:330-350); padding rows still take part in cross attention."""
    g, om, synth = tiny_oracle
    r = synth.make_request(g, 2)
    r.prompt[g.prompt_tokens // 2:] = 0.0
    out = om.predict(r)["action"]
    assert np.isfinite(out).all()


def test_oracle_prefix_state_row_uses_action_rope_position_zero(tiny_oracle):
    """Prefix key row 0 is the state token (cache.cpp:404-412 reads it at index 0)."""
    g, om, synth = tiny_oracle
    r = synth.make_request(g, 3)
    d = om.predict(r, dumps=True)
    assert d["prefix_k"].shape[2] == 1 + g.grid_h * g.grid_w


def test_engine_adapter_library_exports():
    """lib/libwam_b200_adapter.so (B200Engine compiled against the reference's
    engine.h) loads next to libwam_b200.so and exports its harness; no GPU call."""
    import ctypes as C

    adapter = REPO / "wam.cpp_b200" / "lib" / "libwam_b200_adapter.so"
    if not adapter.exists():
        pytest.skip("adapter not built here (needs WAM_REFERENCE_ROOT at build time)")
    import wam_b200

    wam_b200.load()
    lib = C.CDLL(str(adapter))
    for sym in ("wam_b200_adapter_create", "wam_b200_adapter_destroy", "wam_b200_adapter_predict",
                "wam_b200_adapter_reset", "wam_b200_adapter_cfg", "wam_b200_adapter_stats"):
        assert hasattr(lib, sym), sym
