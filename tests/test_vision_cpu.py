"""Vision front-end stage 1 on the CPU: the oracle's image composition
(oracle/vision.cpp) against golden vectors made by the reference's own
compose_and_patchify (tests/golden/make_golden_vision.py), bit for bit."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden" / "vision_compose.npz"


def golden_cases():
    z = np.load(GOLDEN)
    meta = json.loads(bytes(z["meta"]).decode())
    return [(c, z[c["array"]] if "array" in c else None) for c in meta["cases"]]


@pytest.mark.parametrize("case", range(5))
def test_oracle_matches_reference_golden(case):
    import oracle
    from wam_b200.workload import make_views

    c, want = golden_cases()[case]
    views = make_views(c["seed"], [tuple(s) for s in c["sizes"]], c["formats"])
    got = oracle.compose_and_patchify(views, c["width"], c["height"])
    assert got.shape == (12, c["height"] // 2, c["width"] // 2)
    assert hashlib.sha256(got.tobytes()).hexdigest() == c["sha256"]
    if want is not None:
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_oracle_matches_compiled_reference_when_built():
    import oracle
    from wam_b200.workload import make_views

    if not oracle.REF_VISION_LIB.exists():
        pytest.skip("oracle/_ref/libwamref_vision.so not built (make -C oracle ref REF=...)")
    rng = np.random.Generator(np.random.PCG64(5))
    for _ in range(6):
        sizes = [tuple(int(x) for x in rng.integers(3, 200, 2)) for _ in range(3)]
        fmts = [("u8", "f32")[int(x)] for x in rng.integers(0, 2, 3)]
        w, h = (int(x) * 2 for x in rng.integers(4, 60, 2))
        views = make_views(int(rng.integers(1 << 30)), sizes, fmts)
        a = oracle.compose_and_patchify(views, w, h)
        b = oracle.compose_and_patchify(views, w, h, reference=True)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (sizes, fmts, w, h)


def test_oracle_rejects_bad_canvas():
    import oracle
    from wam_b200.workload import make_views

    views = make_views(1, ((8, 8),) * 3)
    with pytest.raises(ValueError):
        oracle.compose_and_patchify(views, 33, 16)


def test_vae_tensor_specs_match_library():
    """The Python spec list (GGUF writers, oracle weights) equals the encoder's
    own (csrc/vae.cu), read through the C ABI without a GPU: 82 tensors, the
    reference's count for the vae component (artifact.cpp:159)."""
    import ctypes as C

    from wam_b200 import load
    from wam_b200.vision import vae_tensor_specs

    lib = load()
    fn = lib.wam_b200_vae_tensor_spec
    fn.restype = C.c_int
    fn.argtypes = [C.c_int, C.c_int, C.c_char_p, C.c_size_t, C.POINTER(C.c_longlong)]
    py = vae_tensor_specs(48)
    assert len(py) == 82
    got = []
    buf = C.create_string_buffer(128)
    shape = (C.c_longlong * 4)()
    i = 0
    while True:
        nd = fn(48, i, buf, 128, shape)
        if nd < 0:
            break
        got.append((buf.value.decode(), tuple(shape[j] for j in range(nd))))
        i += 1
    assert got == py
