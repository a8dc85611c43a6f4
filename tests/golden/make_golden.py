"""Generates tests/golden/reference_host.json from the reference's OWN host code.

Runs only where the reference tree is present: `make -C oracle ref` compiles
src/models/common/scheduler.cpp and src/models/gwp05/semantics.cpp from the
reference sources into oracle/_ref/libwamref.so; this script calls them and
records their outputs (flow-match schedules, visual/action positions,
state normalisation, action post-processing) as golden vectors. The tests pin
the oracle and the engine's host logic to these vectors.

Usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import ctypes as C
import json
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))


def main() -> None:
    subprocess.run(["make", "-C", str(REPO / "oracle"), "ref"], check=True)
    import oracle

    ref = oracle.ref_lib()
    f32p = C.POINTER(C.c_float)
    i32p = C.POINTER(C.c_int32)
    out: dict = {"source": "GigaAI-research/wam.cpp scheduler.cpp + semantics.cpp (compiled)",
                 "schedules": [], "visual_positions": [], "action_positions": [],
                 "normalize_state": [], "postprocess": []}
    for steps, shift in [(10, 1.0), (10, 5.0), (1, 5.0), (4, 3.0), (50, 5.0)]:
        ts = np.zeros(steps, np.float32)
        sig = np.zeros(steps + 1, np.float32)
        assert ref.wamref_schedule(steps, shift, ts.ctypes.data_as(f32p), sig.ctypes.data_as(f32p)) == 0
        out["schedules"].append({"steps": steps, "shift": shift,
                                 "timesteps_bits": ts.view(np.uint32).tolist(),
                                 "sigmas_bits": sig.view(np.uint32).tolist()})
    for gh, gw in [(32, 24), (10, 12), (4, 4), (1, 3)]:
        n = gh * gw
        t, h, w = (np.zeros(n, np.int32) for _ in range(3))
        assert ref.wamref_visual_positions(gh, gw, t.ctypes.data_as(i32p), h.ctypes.data_as(i32p),
                                           w.ctypes.data_as(i32p)) == 0
        out["visual_positions"].append({"grid": [gh, gw], "t": t.tolist(), "h": h.tolist(),
                                        "w": w.tolist()})
    for tokens, state in [(48, 0), (48, 1), (16, 0)]:
        p = np.zeros(tokens + state, np.int32)
        assert ref.wamref_action_positions(tokens, state, p.ctypes.data_as(i32p)) == 0
        out["action_positions"].append({"tokens": tokens, "include_state": state,
                                        "positions": p.tolist()})
    rng = np.random.Generator(np.random.PCG64(7))
    i = np.arange(32, dtype=np.float32)
    q01 = (-1.0 - 0.01 * i).astype(np.float32)
    q99 = (1.0 + 0.02 * i).astype(np.float32)
    q99[5] = q01[5]  # degenerate range exercises the 1e-8 clamp
    for n in (14, 32, 1):
        s = rng.standard_normal(n).astype(np.float32)
        o = np.zeros(32, np.float32)
        assert ref.wamref_normalize_state(s.ctypes.data_as(f32p), n, 32, q01.ctypes.data_as(f32p),
                                          q99.ctypes.data_as(f32p), o.ctypes.data_as(f32p)) == 0
        out["normalize_state"].append({"state": s.tolist(), "q01": q01.tolist(), "q99": q99.tolist(),
                                       "out_bits": o.view(np.uint32).tolist()})
    for steps, real in [(48, 14), (3, 32), (2, 1)]:
        a = rng.standard_normal((steps, 32)).astype(np.float32)
        st = rng.standard_normal(32).astype(np.float32)
        o = np.zeros(steps * real, np.float32)
        assert ref.wamref_postprocess(a.ctypes.data_as(f32p), steps, 32, real,
                                      q01.ctypes.data_as(f32p), q99.ctypes.data_as(f32p),
                                      st.ctypes.data_as(f32p), 32, o.ctypes.data_as(f32p)) == 0
        out["postprocess"].append({"steps": steps, "real": real, "action": a.ravel().tolist(),
                                   "state": st.tolist(), "q01": q01.tolist(), "q99": q99.tolist(),
                                   "out_bits": o.view(np.uint32).tolist()})
    (HERE / "reference_host.json").write_text(json.dumps(out))
    print("wrote", HERE / "reference_host.json")


if __name__ == "__main__":
    main()
