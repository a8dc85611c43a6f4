"""Generates tests/golden/reference_text.json from the reference's OWN
timestep_embedding and relative_position_bucket
(src/models/gwp05/engine/text_encoder.cpp:1-24), compiled by
`make -C oracle ref` into oracle/_ref/libwamref_text.so.

Usage: REF=<reference tree> python tests/golden/make_golden_text.py
"""
from __future__ import annotations

import ctypes as C
import json
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def main() -> None:
    ref = os.environ.get("REF") or os.environ.get("WAM_REFERENCE_ROOT")
    if not ref:
        raise SystemExit("set REF to the reference source tree")
    subprocess.run(["make", "-C", str(REPO / "oracle"), "ref", f"REF={ref}"], check=True)
    lib = C.CDLL(str(REPO / "oracle" / "_ref" / "libwamref_text.so"))
    lib.wamref_relative_bucket.restype = C.c_int
    lib.wamref_relative_bucket.argtypes = [C.c_int, C.c_int, C.c_int]
    lib.wamref_timestep_embedding.argtypes = [C.c_float, C.c_int, C.POINTER(C.c_float)]
    rel = list(range(-1100, 1101))
    out = {"source": "GigaAI-research/wam.cpp engine/text_encoder.cpp:1-24 (compiled)",
           "relative": rel,
           "bucket_32_128": [lib.wamref_relative_bucket(r, 32, 128) for r in rel],
           "timestep_embedding": []}
    for t in (0.0, 1.0, 37.5, 500.0, 999.0, 1000.0):
        v = np.zeros(256, np.float32)
        lib.wamref_timestep_embedding(t, 256, v.ctypes.data_as(C.POINTER(C.c_float)))
        out["timestep_embedding"].append({"t": t, "dim": 256, "bits": v.view(np.uint32).tolist()})
    (HERE / "reference_text.json").write_text(json.dumps(out))
    print("wrote", HERE / "reference_text.json")


if __name__ == "__main__":
    main()
