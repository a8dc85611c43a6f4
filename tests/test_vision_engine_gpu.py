"""Requests carrying camera views instead of a precomputed latent: the
engine's vision front-end (stage 1 + the VAE encoder on the device, the
reference's run_vae path when no latent is given, engine.cpp:260-270).

* bit-identical to encoding the views with the standalone VAE and passing the
  latent (same synthetic weights, same kernels);
* end to end against the CPU oracle chain compose_and_patchify -> VAE ->
  MoT forward: actions within the 5e-2 relative-L2 gate;
* through the reference's Engine vtable (the B200Engine adapter), when built.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED = 20261201


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30))


def _views():
    from wam_b200.workload import make_views

    return make_views(9, ((480, 640), (240, 320), (360, 200)))


@pytest.mark.parametrize("geom_name", ["TINY", "SMALL"])
def test_images_equal_latent_from_standalone_vae(cuda_device, geom_name):
    from oracle import synth
    from wam_b200 import vision
    from wam_b200.engine import Engine, Req

    g = getattr(synth, geom_name)
    r = synth.make_request(g, 3)
    views = _views()
    vae = vision.Vae(g.grid_w * 32, g.grid_h * 32, z_dim=g.vae_z, seed=SEED)
    lat = vae.encode(views)
    e_img = Engine(g, seed=SEED, bias_scale=0.02, prompt_cache=False, vae=True)
    a = e_img.predict(Req(r.state, None, r.prompt, r.noise, images=views))
    e_lat = Engine(g, seed=SEED, bias_scale=0.02, prompt_cache=False)
    b = e_lat.predict(Req(r.state, lat.reshape(-1), r.prompt, r.noise))
    assert np.isfinite(a).all()
    assert np.array_equal(a, b)
    # A batch mixing a latent request and an image request.
    e2 = Engine(g, seed=SEED, bias_scale=0.02, prompt_cache=False, vae=True, max_batch=2)
    out = e2.predict_batch([Req(r.state, lat.reshape(-1), r.prompt, r.noise),
                            Req(r.state, None, r.prompt, r.noise, images=views)])
    assert np.array_equal(out[0], b) and np.array_equal(out[1], b)


def test_images_match_oracle_chain(cuda_device):
    import oracle
    from oracle import synth
    from wam_b200 import vision
    from wam_b200.engine import Engine, Req

    g = synth.TINY
    r = synth.make_request(g, 5)
    views = _views()
    W, H = g.grid_w * 32, g.grid_h * 32
    mean, std = vision.vae_synthetic_stats(g.vae_z)
    pix = oracle.compose_and_patchify(views, W, H)
    lat = oracle.vae_encode(synth.make_vae_weights(SEED, g.vae_z), mean, std, g.vae_z, pix, W, H)
    om = oracle.OracleModel(g, synth.make_weights(g, SEED, bias_scale=0.02))
    r.latent = lat.reshape(-1).astype(np.float32)
    ref = om.predict(r)
    eng = Engine(g, seed=SEED, bias_scale=0.02, prompt_cache=False, vae=True)
    out = eng.predict(Req(r.state, None, r.prompt, r.noise, images=views))
    assert rel_l2(out, ref["action"]) < 5e-2


def test_images_need_vae_engine_and_three_views(cuda_device):
    from oracle import synth
    from wam_b200.engine import Engine, Req

    g = synth.TINY
    r = synth.make_request(g, 5)
    views = _views()
    e = Engine(g, seed=SEED, prompt_cache=False)
    with pytest.raises(RuntimeError, match="vae = 1"):
        e.predict(Req(r.state, None, r.prompt, r.noise, images=views))
    ev = Engine(g, seed=SEED, prompt_cache=False, vae=True)
    with pytest.raises(RuntimeError, match="three input images"):
        ev.predict(Req(r.state, None, r.prompt, r.noise, images=views[:2]))
