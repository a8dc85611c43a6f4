"""The batch-capable serving surface (csrc/batcher.cpp): concurrent callers on
many threads are served as predict_batch calls of several requests, each gets
its own chunk (equal to predict_batch of the same requests), and a bad request
fails alone while the others in its batch succeed."""
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED = 20261201


def test_batcher_concurrent_requests(cuda_device):
    from oracle import synth
    from wam_b200.engine import Batcher, Engine, Req

    g = synth.TINY
    eng = Engine(g, seed=SEED, bias_scale=0.02, prompt_cache=False, max_batch=4)
    reqs = []
    for i in range(12):
        r = synth.make_request(g, 100 + i)
        reqs.append(Req(r.state, r.latent, r.prompt, r.noise))
    # The chunk of a request does not depend on its batch position or batch
    # size (requests are independent), so one batch of 4 gives the reference.
    ref = np.concatenate([eng.predict_batch(reqs[i:i + 4]) for i in range(0, 12, 4)])
    b = Batcher(eng, max_wait_us=20000)
    outs, sizes, errs = [None] * 12, [0] * 12, []
    start = threading.Barrier(12)

    def worker(i):
        try:
            start.wait()
            outs[i], sizes[i] = b.predict(reqs[i])
        except Exception as e:  # noqa: BLE001
            errs.append(e)

    th = [threading.Thread(target=worker, args=(i,)) for i in range(12)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=120)
    assert not errs, errs
    for i in range(12):
        assert outs[i] is not None
        assert np.abs(outs[i] - ref[i]).max() <= 1e-2 * (np.abs(ref[i]).max() + 1e-6), i
    nb, nr = b.counts()
    assert nr == 12 and nb < 12 and max(sizes) > 1
    b.close()


def test_batcher_bad_request_fails_alone(cuda_device):
    from oracle import synth
    from wam_b200.engine import Batcher, Engine, Req

    g = synth.TINY
    eng = Engine(g, seed=SEED, bias_scale=0.02, prompt_cache=False, max_batch=4)
    good = [synth.make_request(g, 200 + i) for i in range(3)]
    bad = synth.make_request(g, 300)
    st = np.array(bad.state, np.float32)
    st[0] = np.nan
    reqs = [Req(r.state, r.latent, r.prompt, r.noise) for r in good] + [
        Req(st, bad.latent, bad.prompt, bad.noise)]
    b = Batcher(eng, max_wait_us=50000)
    res = [None] * 4
    start = threading.Barrier(4)

    def worker(i):
        start.wait()
        try:
            res[i] = b.predict(reqs[i])[0]
        except RuntimeError as e:
            res[i] = e

    th = [threading.Thread(target=worker, args=(i,)) for i in range(4)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=120)
    assert isinstance(res[3], RuntimeError) and "NaN" in str(res[3])
    for i in range(3):
        assert isinstance(res[i], np.ndarray) and np.isfinite(res[i]).all()
    b.close()
