"""Requests carrying prompt token ids instead of a precomputed embedding: the
engine's resident UMT5 encoder (the reference's resident language-encoder
policy; run_t5, text_encoder.cpp:112-204) feeding the prompt projection.

* bit-identical to encoding the tokens with the standalone TextEncoder and
  passing the embedding (same synthetic weights, same kernels);
* the projected-prompt cache keyed on the token ids (hit on a repeat);
* end to end against the CPU oracle chain UMT5 -> MoT forward (5e-2 gate);
* the reference's mask checks through the engine.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED = 20261201
T5_VOCAB, T5_FFN, T5_LAYERS = 1000, 256, 2


def _geoms():
    from oracle import synth
    from wam_b200.text import T5Geometry

    g = synth.TINY
    tg = T5Geometry(vocab=T5_VOCAB, hidden=g.text_dim, ffn=T5_FFN, heads=g.text_dim // 64,
                    head_dim=64, layers=T5_LAYERS, max_tokens=g.prompt_tokens)
    return g, tg


def _engine(**kw):
    from wam_b200.engine import Engine

    g, _ = _geoms()
    return Engine(g, seed=SEED, bias_scale=0.02, t5=True, t5_vocab=T5_VOCAB, t5_ffn=T5_FFN,
                  t5_layers=T5_LAYERS, **kw)


def test_tokens_equal_embedding_from_standalone_encoder(cuda_device):
    from oracle import synth
    from wam_b200.engine import Engine, Req
    from wam_b200.text import TextEncoder

    g, tg = _geoms()
    r = synth.make_request(g, 4)
    tok = np.random.default_rng(2).integers(0, T5_VOCAB, 11).astype(np.int32)
    emb = TextEncoder(tg, seed=SEED).encode(tok)
    a = _engine(prompt_cache=False).predict(Req(r.state, r.latent, None, r.noise, tokens=tok))
    b = Engine(g, seed=SEED, bias_scale=0.02, prompt_cache=False).predict(
        Req(r.state, r.latent, emb, r.noise))
    assert np.isfinite(a).all()
    assert np.array_equal(a, b)


def test_token_prompt_cache(cuda_device):
    from oracle import synth
    from wam_b200.engine import Req

    g, _ = _geoms()
    r = synth.make_request(g, 4)
    tok = np.random.default_rng(2).integers(0, T5_VOCAB, 11).astype(np.int32)
    e = _engine(prompt_cache=True)
    a, s1 = e.predict(Req(r.state, r.latent, None, r.noise, tokens=tok), stats=True)
    b, s2 = e.predict(Req(r.state, r.latent, None, r.noise, tokens=tok), stats=True)
    assert s1["prompt_cache_hit"] == 0 and s2["prompt_cache_hit"] == 1
    assert np.array_equal(a, b)
    tok2 = tok.copy()
    tok2[3] = (tok2[3] + 1) % T5_VOCAB
    c, s3 = e.predict(Req(r.state, r.latent, None, r.noise, tokens=tok2), stats=True)
    assert s3["prompt_cache_hit"] == 0 and not np.array_equal(a, c)
    # The same tokens with a mask of ones over a padded tail are the same prompt.
    pad = np.concatenate([tok, np.zeros(5, np.int32)])
    mask = np.array([1] * 11 + [0] * 5, np.int32)
    d, s4 = e.predict(Req(r.state, r.latent, None, r.noise, tokens=pad, mask=mask), stats=True)
    e.predict(Req(r.state, r.latent, None, r.noise, tokens=tok))
    d2, s5 = e.predict(Req(r.state, r.latent, None, r.noise, tokens=pad, mask=mask), stats=True)
    assert s5["prompt_cache_hit"] == 1 and np.array_equal(d, a) and np.array_equal(d2, a)


def test_tokens_match_oracle_chain(cuda_device):
    import oracle
    from oracle import synth
    from wam_b200.engine import Req

    g, tg = _geoms()
    r = synth.make_request(g, 6)
    tok = np.random.default_rng(9).integers(0, T5_VOCAB, 13).astype(np.int32)
    emb = oracle.t5_encode(synth.make_t5_weights(SEED, tg), tg, tok, tg.max_tokens)
    om = oracle.OracleModel(g, synth.make_weights(g, SEED, bias_scale=0.02))
    r.prompt = emb
    ref = om.predict(r)
    out = _engine(prompt_cache=False).predict(Req(r.state, r.latent, None, r.noise, tokens=tok))
    err = float(np.linalg.norm(out - ref["action"]) / np.linalg.norm(ref["action"]))
    assert err < 5e-2, err


def test_token_request_checks(cuda_device):
    from oracle import synth
    from wam_b200.engine import Engine, Req

    g, _ = _geoms()
    r = synth.make_request(g, 4)
    tok = np.arange(8, dtype=np.int32)
    with pytest.raises(RuntimeError, match="t5 = 1"):
        Engine(g, seed=SEED).predict(Req(r.state, r.latent, None, r.noise, tokens=tok))
    e = _engine(prompt_cache=False)
    with pytest.raises(RuntimeError, match="contiguous valid prefix"):
        e.predict(Req(r.state, r.latent, None, r.noise, tokens=tok,
                      mask=np.array([1, 0, 1, 1, 1, 1, 1, 1], np.int32)))
    with pytest.raises(RuntimeError, match="outside"):
        e.predict(Req(r.state, r.latent, None, r.noise,
                      tokens=np.zeros(g.prompt_tokens + 1, np.int32)))
    with pytest.raises(RuntimeError, match="vocabulary"):
        e.predict(Req(r.state, r.latent, None, r.noise, tokens=np.full(4, T5_VOCAB, np.int32)))
