"""Vision front-end stage 1 on the B200 (csrc/vision.cu through the C ABI):
bit-identical to the oracle (itself pinned to the reference's own
compose_and_patchify by golden vectors), from device views and through the
host-image Preprocessor, with the reference's argument checks."""
import hashlib

import numpy as np
import pytest
import torch

from test_vision_cpu import golden_cases

pytestmark = pytest.mark.gpu


def _dev(views):
    return [torch.from_numpy(v).cuda() for v in views]


@pytest.mark.parametrize("case", range(5))
def test_preprocess_matches_reference_golden(cuda_device, case):
    from wam_b200 import vision
    from wam_b200.workload import make_views

    c, want = golden_cases()[case]
    views = make_views(c["seed"], [tuple(s) for s in c["sizes"]], c["formats"])
    got = vision.preprocess(_dev(views), c["width"], c["height"]).cpu().numpy()
    assert hashlib.sha256(got.tobytes()).hexdigest() == c["sha256"]
    if want is not None:
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("seed,sizes,fmts,w,h", [
    (21, ((480, 640), (480, 640), (480, 640)), ("u8", "u8", "u8"), 768, 1024),   # config 2
    (22, ((1080, 1920), (720, 1280), (2160, 3840)), ("u8", "u8", "u8"), 256, 160),  # 8-15x down
    (23, ((5, 3), (2, 2), (1, 1)), ("f32", "u8", "f32"), 64, 32),               # extreme up
    (24, ((300, 301), (97, 33), (33, 97)), ("f32", "f32", "u8"), 2, 2),           # 1-pixel cells
])
def test_preprocess_matches_oracle(cuda_device, seed, sizes, fmts, w, h):
    import oracle
    from wam_b200 import vision
    from wam_b200.workload import make_views

    views = make_views(seed, sizes, fmts)
    want = oracle.compose_and_patchify(views, w, h)
    got = vision.preprocess(_dev(views), w, h).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_preprocessor_host_images_grow_and_reuse(cuda_device):
    import oracle
    from wam_b200 import vision
    from wam_b200.workload import make_views

    p = vision.Preprocessor(0)
    for seed, sizes, w, h in [(31, ((20, 30),) * 3, 64, 64), (32, ((480, 640),) * 3, 768, 1024),
                              (33, ((10, 10),) * 3, 32, 32)]:
        views = make_views(seed, sizes)
        got = p(views, w, h).cpu().numpy()
        want = oracle.compose_and_patchify(views, w, h)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    p.close()


def test_preprocess_argument_checks(cuda_device):
    from wam_b200 import vision
    from wam_b200.workload import make_views

    p = vision.Preprocessor(0)
    views = make_views(41, ((8, 8),) * 3)
    with pytest.raises(RuntimeError, match="three input images"):
        p(views[:2], 16, 16)
    with pytest.raises(RuntimeError, match="positive and even"):
        p(views, 15, 16)
    with pytest.raises(RuntimeError, match="positive and even"):
        vision.preprocess(_dev(views), 16, 6 + 1)
    bad = [views[0], np.zeros((0, 4, 3), np.uint8), views[2]]
    with pytest.raises(RuntimeError, match="invalid image 1"):
        p(bad, 16, 16)
