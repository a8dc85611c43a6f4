"""GGUF artifacts through the engine's loader (wam_b200_create with an
artifact path): a TINY artifact written with the gguf-py writer from the
synthetic weights must give bit-identical actions to the engine's own
synthetic weights, in BF16 and with Q8_0 linear weights (GGML type 8, made by
gguf-py's quantiser, which the device quantiser matches bit for bit)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
gguf = pytest.importorskip("gguf")
from gguf_fixture import SEED, write_artifact  # noqa: E402


@pytest.mark.parametrize("q8", [False, True])
def test_gguf_artifact_matches_synthetic(cuda_device, tmp_path, q8):
    from oracle import synth
    from wam_b200.engine import Engine, Req

    g = synth.TINY
    path = tmp_path / ("tiny_q8.gguf" if q8 else "tiny_bf16.gguf")
    write_artifact(path, g, q8)
    r = synth.make_request(g, 17)
    req = Req(r.state, r.latent, r.prompt, r.noise)
    fmt = "q8_0" if q8 else "bf16"
    a = Engine(artifact=str(path), prompt_cache=False, weights=fmt).predict(req)
    b = Engine(g, seed=SEED, bias_scale=0.02, prompt_cache=False, weights=fmt).predict(req)
    assert np.isfinite(a).all()
    assert np.array_equal(a, b)


def test_q8_policy_artifact_matches_device_quantiser(cuda_device, tmp_path):
    """A mot-q8_0-v1 artifact made by wam_b200.artifact.convert from a BF16
    artifact gives the same actions, bit for bit, as the engine quantising the
    synthetic weights on the device; the policy selects the Q8_0 path even when
    the caller asks for BF16."""
    from oracle import synth
    from wam_b200 import artifact
    from wam_b200.engine import Engine, Req

    g = synth.TINY
    src, dst = tmp_path / "bf16.gguf", tmp_path / "q8.gguf"
    write_artifact(src, g, q8=False, policy=artifact.BF16_POLICY_ID)
    artifact.convert(src, dst)
    r = synth.make_request(g, 23)
    req = Req(r.state, r.latent, r.prompt, r.noise)
    a = Engine(artifact=str(dst), prompt_cache=False, weights="bf16").predict(req)
    b = Engine(g, seed=SEED, bias_scale=0.02, prompt_cache=False, weights="q8_0").predict(req)
    c = Engine(artifact=str(src), prompt_cache=False, weights="bf16").predict(req)
    assert np.isfinite(a).all()
    assert np.array_equal(a, b)
    assert not np.array_equal(a, c)


@pytest.mark.parametrize("q8,policy,match", [
    (False, "mot-q8_0-v1", "does not allow"),
    (True, "mot-vae-bf16-qkv-v1", "does not allow"),
    (False, "mot-bf16-v1", "unsupported weight policy"),
])
def test_engine_rejects_policy_violations(cuda_device, tmp_path, q8, policy, match):
    from oracle import synth
    from wam_b200.engine import Engine

    p = tmp_path / "bad.gguf"
    write_artifact(p, synth.TINY, q8=q8, policy=policy)
    with pytest.raises(RuntimeError, match=match):
        Engine(artifact=str(p), prompt_cache=False)
