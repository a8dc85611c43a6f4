"""GGUF artifact tooling for the Q8_0 weight policy ``mot-q8_0-v1``.

The reference defines its weight policies in ``scripts/common/gwp05_gguf.py``
(``POLICIES``, :19-41), writes them with ``scripts/convert/convert_gwp05.py`` and
checks them with ``scripts/inspect/inspect_gguf.py`` (``_policy`` :60-75,
``validate_reader`` :78-200). None of them knows Q8_0: its stored dtypes are F32
and BF16 only (``DTYPE_BYTES``, :14; ``artifact.cpp:129-139``). This module is the
Q8_0 counterpart of those three pieces:

* ``POLICY_Q8`` -- the policy entry a maintainer adds next to
  ``mot-vae-bf16-qkv-v1``: packed self-attention QKV, every ``gwp.*`` linear
  weight whose GGUF rows (``ne[0]``) are whole 32-value blocks stored as GGML
  type 8 (Q8_0: an fp16 scale ``d`` and 32 int8 ``q`` per block, value ``q*d``),
  everything else as in the BF16 policy;
* ``convert(src, dst)`` -- re-quantises a ``mot-vae-bf16-qkv-v1`` artifact (or an
  unlabelled BF16 one) into ``mot-q8_0-v1``, one tensor at a time, with the
  ``gguf`` package's own Q8_0 quantiser applied to the BF16 values widened to
  F32 (the same rule the engine's device quantiser follows bit for bit);
* ``inspect(path)`` -- the ``validate_reader`` of the policy: architecture,
  policy keys, per-tensor dtype rule, component telemetry.

The engine (``wam_b200_create`` with an artifact path) accepts both policies
and rejects a file whose tensors break the policy it names.

Command line::

    python -m wam_b200.artifact convert SRC.gguf DST.gguf
    python -m wam_b200.artifact inspect ART.gguf [--expect-policy mot-q8_0-v1]
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path
from typing import Any

import numpy as np

ARCH = "gwp05"
# The reference's converter revision string (gwp05_gguf.py:11); the Q8_0 pass
# appends its own suffix so an inspector can tell the two writers apart.
CONVERTER_REVISION = "gwp05-native-bf16-v1+b200-q8_0-v1"
BF16_POLICY_ID = "mot-vae-bf16-qkv-v1"
Q8_POLICY_ID = "mot-q8_0-v1"
POLICY_Q8: dict[str, Any] = {
    "id": Q8_POLICY_ID,
    "source": {"gwp": "BF16", "t5": "BF16", "vae": "BF16", "stats": "F32"},
    # gwp: Q8_0 for linear weights with whole 32-value rows, BF16 otherwise.
    "stored": {"gwp": "Q8_0|BF16", "t5": "BF16", "vae": "BF16", "stats": "F32"},
    "pack_self_qkv": True,
}
SOURCE_POLICIES = ("", BF16_POLICY_ID)
_NORM_GAINS = (".qn.weight", ".kn.weight", "ca_norm.weight")
_POLICY_KEYS = ("weight_policy", "conversion_policy", "converter_revision")
_STAT_FIELDS = ("source_dtype", "stored_dtype", "tensor_count", "elements",
                "source_bytes", "stored_bytes")


class ContractError(ValueError):
    """An artifact that breaks the policy it names (inspect_gguf.py ContractError)."""


def _gguf():
    try:
        import gguf
    except ModuleNotFoundError as exc:  # same message as inspect_gguf.py:13-17
        raise SystemExit("missing Python package 'gguf'") from exc
    return gguf


def q8_tensor(name: str, ne: tuple[int, ...]) -> bool:
    """Whether ``mot-q8_0-v1`` stores this tensor as Q8_0: a ``gwp.*`` linear
    weight (any ``.weight`` except the q/k RMSNorm and cross-attention LayerNorm
    gains) of at least two dimensions whose rows ``ne[0]`` are whole 32-value
    blocks. ``gwp.patch.weight`` (``ne[0] = 2``, the 2x2 kernel) stays BF16; the
    engine quantises it at load, flattened to rows of ``4 * vae_z_dim``."""
    return (name.startswith("gwp.") and name.endswith(".weight")
            and not name.endswith(_NORM_GAINS) and len(ne) >= 2 and ne[0] % 32 == 0)


def component(name: str) -> str:
    if name.startswith("gwp."):
        return "gwp"
    if name.startswith("t5."):
        return "t5"
    if name.startswith("vae."):
        return "vae"
    return "stats"


def _field(reader, key: str, default: Any = None) -> Any:
    f = reader.get_field(key)
    return default if f is None else f.contents()


def _bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


def quantize_bf16_rows(u16: np.ndarray) -> np.ndarray:
    """Q8_0 blocks (uint8, last axis 34 bytes per 32 values) of BF16 bits, the
    values widened to F32 exactly and quantised by ``gguf.quants`` (gguf-py's
    ``quantize_q8_0``: ``d = max|x| / 127``, ``q = round(x / d)``)."""
    gguf = _gguf()
    return gguf.quants.quantize(_bf16_to_f32(u16), gguf.GGMLQuantizationType.Q8_0)


def _copy_kv(reader, writer, skip: set[str]) -> None:
    gguf = _gguf()
    V = gguf.GGUFValueType
    for key, f in reader.fields.items():
        if key.startswith("GGUF.") or key == "general.architecture" or key in skip:
            continue
        vtype = f.types[0]
        sub = f.types[1] if vtype == V.ARRAY and len(f.types) > 1 else None
        writer.add_key_value(key, f.contents(), vtype, sub)


def convert(src: str | Path, dst: str | Path) -> dict[str, Any]:
    """Write ``dst`` as the ``mot-q8_0-v1`` re-quantisation of ``src`` (a BF16
    artifact, policy ``mot-vae-bf16-qkv-v1`` or unlabelled). Streams one tensor
    at a time; returns the component telemetry written into the metadata."""
    gguf = _gguf()
    reader = gguf.GGUFReader(str(src), "r")
    if _field(reader, "gwp05.architecture") != ARCH:
        raise ContractError("source is not a gwp05 artifact")
    policy = _field(reader, "gwp05.weight_policy", "")
    if policy not in SOURCE_POLICIES:
        raise ContractError(f"source policy {policy!r} is not a BF16 packed-QKV policy")
    T = gguf.GGMLQuantizationType
    plan = []
    stats = {c: {"source_dtype": POLICY_Q8["source"][c], "stored_dtype": POLICY_Q8["stored"][c],
                 "tensor_count": 0, "elements": 0, "source_bytes": 0, "stored_bytes": 0}
             for c in ("gwp", "t5", "vae", "stats")}
    for t in reader.tensors:
        ne = tuple(int(x) for x in t.shape)
        q8 = q8_tensor(t.name, ne)
        if q8 and t.tensor_type != T.BF16:
            raise ContractError(f"{t.name}: source dtype {t.tensor_type.name}, expected BF16")
        nbytes = int(t.n_elements) // 32 * 34 if q8 else int(t.n_bytes)
        plan.append((t, q8, nbytes))
        s = stats[component(t.name)]
        s["tensor_count"] += 1
        s["elements"] += int(t.n_elements)
        s["source_bytes"] += int(t.n_bytes)
        s["stored_bytes"] += nbytes

    w = gguf.GGUFWriter(str(dst), ARCH)
    skip = {f"gwp05.{k}" for k in _POLICY_KEYS}
    skip |= {f"gwp05.{c}_{f}" for c in stats for f in _STAT_FIELDS}
    _copy_kv(reader, w, skip)
    for k in ("weight_policy", "conversion_policy"):
        w.add_string(f"gwp05.{k}", Q8_POLICY_ID)
    w.add_string("gwp05.converter_revision", CONVERTER_REVISION)
    for c, s in stats.items():
        for f in _STAT_FIELDS:
            if isinstance(s[f], str):
                w.add_string(f"gwp05.{c}_{f}", s[f])
            else:
                w.add_uint64(f"gwp05.{c}_{f}", int(s[f]))
    for t, q8, nbytes in plan:
        np_shape = tuple(reversed([int(x) for x in t.shape]))
        raw = t.tensor_type
        if q8:
            byte_shape = np_shape[:-1] + (np_shape[-1] // 32 * 34,)
            w.add_tensor_info(t.name, byte_shape, np.dtype(np.uint8), nbytes, T.Q8_0)
        else:
            w.add_tensor_info(t.name, t.data.shape, t.data.dtype, nbytes,
                              None if t.data.dtype != np.uint8 else raw)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_ti_data_to_file()
    for t, q8, nbytes in plan:
        if q8:
            u16 = np.ascontiguousarray(t.data).view(np.uint16)
            blocks = quantize_bf16_rows(u16)
            assert blocks.nbytes == nbytes
            w.write_tensor_data(blocks)
        else:
            w.write_tensor_data(np.ascontiguousarray(t.data))
    w.close()
    return stats


def inspect(path: str | Path, expected_policy: str | None = None) -> dict[str, Any]:
    """Validate an artifact against the policy it names (the ``validate_reader``
    of ``mot-q8_0-v1`` and ``mot-vae-bf16-qkv-v1``); raises ContractError."""
    gguf = _gguf()
    reader = gguf.GGUFReader(str(path), "r")
    if _field(reader, "gwp05.architecture") != ARCH:
        raise ContractError("artifact architecture is not gwp05")
    policy = _field(reader, "gwp05.weight_policy", "")
    if policy and _field(reader, "gwp05.conversion_policy", policy) != policy:
        raise ContractError("gwp05.weight_policy differs from conversion_policy")
    if policy not in (Q8_POLICY_ID, BF16_POLICY_ID, ""):
        raise ContractError(f"unsupported weight policy: {policy}")
    if expected_policy is not None and policy != expected_policy:
        raise ContractError(f"policy {policy!r}, expected {expected_policy!r}")
    q8_policy = policy == Q8_POLICY_ID
    if q8_policy and _field(reader, "gwp05.converter_revision") != CONVERTER_REVISION:
        raise ContractError("unsupported converter revision")
    T = gguf.GGMLQuantizationType
    comps: dict[str, dict[str, int]] = {}
    names = set()
    for t in reader.tensors:
        if t.name in names:
            raise ContractError(f"duplicate tensor name {t.name}")
        names.add(t.name)
        ne = tuple(int(x) for x in t.shape)
        c = component(t.name)
        if c == "stats":
            want = {T.F32}
        elif q8_policy and q8_tensor(t.name, ne):
            want = {T.Q8_0}
        elif policy:
            want = {T.BF16}
        else:  # unlabelled fixture: BF16, or Q8_0 where the row rule allows it
            want = {T.BF16, T.Q8_0} if q8_tensor(t.name, ne) else {T.BF16}
        if t.tensor_type not in want:
            raise ContractError(f"{t.name}: dtype {t.tensor_type.name}, expected "
                                f"{'/'.join(sorted(x.name for x in want))}")
        s = comps.setdefault(c, {"tensor_count": 0, "elements": 0, "stored_bytes": 0,
                                 "q8_tensors": 0})
        s["tensor_count"] += 1
        s["elements"] += int(t.n_elements)
        s["stored_bytes"] += int(t.n_bytes)
        s["q8_tensors"] += int(t.tensor_type == T.Q8_0)
    if q8_policy:
        for c, s in comps.items():
            for f in ("tensor_count", "elements", "stored_bytes"):
                got = _field(reader, f"gwp05.{c}_{f}")
                if got != s[f]:
                    raise ContractError(f"gwp05.{c}_{f}: metadata {got!r}, computed {s[f]!r}")
    for k in ("gwp05.hidden", "gwp05.n_layers", "gwp05.n_heads", "gwp05.head_dim"):
        if reader.get_field(k) is None:
            raise ContractError(f"missing metadata: {k}")
    return {"architecture": ARCH, "policy": policy or "unlabelled", "components": comps,
            "tensor_count": len(reader.tensors),
            "layers": int(_field(reader, "gwp05.n_layers"))}


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("convert", help="re-quantise a BF16 artifact to mot-q8_0-v1")
    c.add_argument("src", type=Path)
    c.add_argument("dst", type=Path)
    i = sub.add_parser("inspect", help="validate an artifact against its policy")
    i.add_argument("artifact", type=Path)
    i.add_argument("--expect-policy", choices=(Q8_POLICY_ID, BF16_POLICY_ID))
    a = ap.parse_args(argv)
    try:
        if a.cmd == "convert":
            if a.dst.exists():
                raise ContractError(f"refusing to overwrite {a.dst}")
            report = {"valid": True, "components": convert(a.src, a.dst)}
            report.update(inspect(a.dst, Q8_POLICY_ID))
        else:
            report = {"valid": True, **inspect(a.artifact, a.expect_policy)}
    except (ContractError, OSError, ValueError) as exc:
        report = {"valid": False, "error": str(exc)}
    print(json.dumps(report, indent=2, sort_keys=True))
    return 0 if report["valid"] else 1


if __name__ == "__main__":
    sys.exit(main())
