"""B200Engine behind the reference's Engine interface
(src/models/gwp05/engine/engine.h:142-155), compiled against the reference's
own engine.h into lib/libwam_b200_adapter.so. The harness functions hold an
Engine* and call predict()/reset() through its vtable, as the model layer does
(src/models/gwp05/model.cpp:221-251).

Checked: Engine::cfg is filled (real_state_dim included, so predict accepts a
state); predict through the base class equals the C ABI engine's chunk bit for
bit and the CPU oracle within 5e-2 relative-L2; reset() keeps it usable; a
NaN state gives the reference's failure value, an empty vector.
"""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ADAPTER = Path(__file__).resolve().parents[1] / "wam.cpp_b200" / "lib" / "libwam_b200_adapter.so"
SEED = 20261203


def _lib():
    import wam_b200

    wam_b200.load()  # libwam_b200.so first (the adapter links to it)
    if not ADAPTER.exists():
        pytest.fail(f"{ADAPTER} not built (python wam.cpp_b200/build.py --reference <tree>)")
    lib = C.CDLL(str(ADAPTER))
    f32p = C.POINTER(C.c_float)
    lib.wam_b200_adapter_create.restype = C.c_void_p
    lib.wam_b200_adapter_create.argtypes = [C.c_void_p]
    lib.wam_b200_adapter_destroy.argtypes = [C.c_void_p]
    lib.wam_b200_adapter_predict.restype = C.c_longlong
    lib.wam_b200_adapter_predict.argtypes = [C.c_void_p, f32p, f32p, C.c_int, f32p, C.c_int, f32p,
                                             f32p, C.c_longlong]
    lib.wam_b200_adapter_reset.argtypes = [C.c_void_p]
    lib.wam_b200_adapter_cfg.restype = C.c_longlong
    lib.wam_b200_adapter_cfg.argtypes = [C.c_void_p, C.c_char_p]
    lib.wam_b200_adapter_stats.argtypes = [C.c_void_p, f32p]
    return lib


def _options(geom):
    from wam_b200._lib_engine import Options
    from wam_b200.engine import geometry_struct

    o = Options()
    o.struct_size = C.sizeof(Options)
    o.synthetic_geometry = geometry_struct(geom)
    o.synthetic_seed = SEED
    o.synthetic_bias_scale = 0.02
    o.max_batch = 1
    o.use_cuda_graphs = 1
    o.prompt_cache = 1
    return o


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _predict(lib, e, r, geom):
    out = np.zeros(geom.action_chunk * geom.real_action_dim, np.float32)
    st = np.ascontiguousarray(r.state, np.float32)
    lat = np.ascontiguousarray(r.latent, np.float32)
    pr = np.ascontiguousarray(r.prompt, np.float32)
    nz = np.ascontiguousarray(r.noise, np.float32)
    n = lib.wam_b200_adapter_predict(e, _fp(st), _fp(lat), lat.size, _fp(pr), pr.shape[0], _fp(nz),
                                     _fp(out), out.size)
    return out[:n].reshape(-1, geom.real_action_dim) if n > 0 else np.zeros((0,), np.float32)


def test_engine_vtable_predict_reset(cuda_device):
    import oracle
    from oracle import synth
    from wam_b200.engine import Engine, Req

    lib = _lib()
    geom = synth.TINY
    o = _options(geom)
    e = lib.wam_b200_adapter_create(C.byref(o))
    assert e, "create_b200_synthetic returned nullptr"
    try:
        assert lib.wam_b200_adapter_cfg(e, b"real_state_dim") == geom.real_state_dim
        assert lib.wam_b200_adapter_cfg(e, b"real_action_dim") == geom.real_action_dim
        assert lib.wam_b200_adapter_cfg(e, b"n_full") == 1 + geom.visual_tokens + geom.action_chunk
        assert lib.wam_b200_adapter_cfg(e, b"n_q_heads") == geom.heads
        assert lib.wam_b200_adapter_cfg(e, b"max_state_dim") == geom.action_dim
        r = synth.make_request(geom, 21)
        got = _predict(lib, e, r, geom)
        assert got.shape == (geom.action_chunk, geom.real_action_dim)
        stats = (C.c_float * 3)()
        lib.wam_b200_adapter_stats(e, stats)
        assert stats[0] > 0 and stats[1] > 0 and stats[2] > 0
        direct = Engine(geom, seed=SEED, bias_scale=0.02).predict(
            Req(r.state, r.latent, r.prompt, r.noise))
        assert np.array_equal(got, direct)
        ref = oracle.OracleModel(geom, None, seed=SEED, bias_scale=0.02).predict(r)["action"]
        err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
        assert err < 5e-2, f"action rel-L2 {err:.3e} vs oracle"
        lib.wam_b200_adapter_reset(e)
        again = _predict(lib, e, r, geom)
        assert np.array_equal(again, got)
        bad = synth.Request(r.state.copy(), r.latent, r.prompt, r.noise)
        bad.state[0] = np.nan
        assert _predict(lib, e, bad, geom).size == 0  # the reference's failure value: {}
        assert np.array_equal(_predict(lib, e, r, geom), got)  # usable after a failure
    finally:
        lib.wam_b200_adapter_destroy(e)


def test_engine_vtable_predict_from_images(cuda_device):
    """EngineInputsView with three camera views and no precomputed latent: the
    adapter hands the views to the engine's vision front-end; the chunk equals
    the C ABI engine's from the same views, bit for bit."""
    from oracle import synth
    from wam_b200.engine import Engine, Req
    from wam_b200.workload import make_views

    lib = _lib()
    u8pp = C.POINTER(C.c_ubyte) * 3
    lib.wam_b200_adapter_predict_images.restype = C.c_longlong
    lib.wam_b200_adapter_predict_images.argtypes = [
        C.c_void_p, C.POINTER(C.c_float), u8pp, C.POINTER(C.c_int), C.POINTER(C.c_int),
        C.POINTER(C.c_float), C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_float), C.c_longlong]
    g = synth.TINY
    o = _options(g)
    o.vae = 1
    e = lib.wam_b200_adapter_create(C.byref(o))
    assert e
    r = synth.make_request(g, 8)
    views = make_views(4, ((480, 640), (240, 320), (200, 300)))
    ptrs = u8pp(*[v.ctypes.data_as(C.POINTER(C.c_ubyte)) for v in views])
    ws = (C.c_int * 3)(*[v.shape[1] for v in views])
    hs = (C.c_int * 3)(*[v.shape[0] for v in views])
    out = np.zeros(g.action_chunk * g.real_action_dim, np.float32)
    st = np.ascontiguousarray(r.state, np.float32)
    pr = np.ascontiguousarray(r.prompt, np.float32)
    nz = np.ascontiguousarray(r.noise, np.float32)
    n = lib.wam_b200_adapter_predict_images(e, _fp(st), ptrs, ws, hs, _fp(pr), pr.shape[0],
                                            _fp(nz), _fp(out), out.size)
    assert n == out.size
    ref = Engine(g, seed=SEED, bias_scale=0.02, prompt_cache=True, vae=True).predict(
        Req(r.state, None, r.prompt, r.noise, images=views))
    assert np.array_equal(out.reshape(ref.shape), ref)
    lib.wam_b200_adapter_destroy(e)


def test_engine_vtable_predict_from_tokens(cuda_device):
    """EngineInputsView with prompt token ids (and a padded mask) and no
    precomputed embedding: the adapter reports the resident language-encoder
    policy and its chunk equals the C ABI engine's from the same tokens."""
    from oracle import synth
    from wam_b200.engine import Engine, Req

    lib = _lib()
    i32p = C.POINTER(C.c_int32)
    lib.wam_b200_adapter_predict_tokens.restype = C.c_longlong
    lib.wam_b200_adapter_predict_tokens.argtypes = [
        C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_float), C.c_int, i32p, C.c_int, i32p,
        C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_float), C.c_longlong]
    g = synth.TINY
    o = _options(g)
    o.t5, o.t5_vocab, o.t5_ffn, o.t5_layers = 1, 1000, 256, 2
    e = lib.wam_b200_adapter_create(C.byref(o))
    assert e
    r = synth.make_request(g, 8)
    tok = np.concatenate([np.random.default_rng(1).integers(0, 1000, 9), np.zeros(4)]).astype(np.int32)
    mask = np.array([1] * 9 + [0] * 4, np.int32)
    out = np.zeros(g.action_chunk * g.real_action_dim, np.float32)
    st = np.ascontiguousarray(r.state, np.float32)
    lat = np.ascontiguousarray(r.latent, np.float32)
    nz = np.ascontiguousarray(r.noise, np.float32)
    n = lib.wam_b200_adapter_predict_tokens(e, _fp(st), _fp(lat), lat.size,
                                            tok.ctypes.data_as(i32p), tok.size,
                                            mask.ctypes.data_as(i32p), mask.size, _fp(nz),
                                            _fp(out), out.size)
    assert n == out.size
    ref = Engine(g, seed=SEED, bias_scale=0.02, t5=True, t5_vocab=1000, t5_ffn=256,
                 t5_layers=2).predict(Req(r.state, r.latent, None, r.noise, tokens=tok[:9]))
    assert np.array_equal(out.reshape(ref.shape), ref)
    lib.wam_b200_adapter_destroy(e)
