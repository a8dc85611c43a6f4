"""The Q8_0 artifact policy tooling (wam_b200.artifact): conversion of a BF16
artifact to mot-q8_0-v1 and its inspection, checked against the gguf package's
own Q8_0 codec (gguf.quants), on the CPU."""
import numpy as np
import pytest

gguf = pytest.importorskip("gguf")
from gguf import quants  # noqa: E402
from gguf_fixture import write_artifact  # noqa: E402


@pytest.fixture(scope="module")
def converted(tmp_path_factory):
    from oracle import synth
    from wam_b200 import artifact

    d = tmp_path_factory.mktemp("art")
    src, dst = d / "bf16.gguf", d / "q8.gguf"
    write_artifact(src, synth.TINY, q8=False, policy=artifact.BF16_POLICY_ID)
    stats = artifact.convert(src, dst)
    return src, dst, stats


def test_convert_quantises_every_linear_weight(converted):
    from wam_b200 import artifact

    src, dst, _ = converted
    rs, rd = gguf.GGUFReader(str(src)), gguf.GGUFReader(str(dst))
    by_name = {t.name: t for t in rd.tensors}
    assert [t.name for t in rs.tensors] == [t.name for t in rd.tensors]
    n_q8 = 0
    for t in rs.tensors:
        o = by_name[t.name]
        assert list(o.shape) == list(t.shape)
        ne = tuple(int(x) for x in t.shape)
        if artifact.q8_tensor(t.name, ne):
            n_q8 += 1
            assert o.tensor_type == gguf.GGMLQuantizationType.Q8_0
            f32 = (np.ascontiguousarray(t.data).view(np.uint16).astype(np.uint32) << 16).view(np.float32)
            want = quants.quantize(f32, gguf.GGMLQuantizationType.Q8_0)
            assert np.array_equal(np.asarray(o.data), want)
            deq = quants.dequantize(np.asarray(o.data), gguf.GGMLQuantizationType.Q8_0)
            # Q8_0: q = round(x / d), d = max|x| / 127 stored as fp16 (d16), so
            # |x - q d16| <= d / 2 + 127 |d16 - d| per block.
            blk = f32.reshape(-1, 32)
            d = np.abs(blk).max(axis=1, keepdims=True) / 127
            d16 = d.astype(np.float16).astype(np.float32)
            bound = d * 0.5 + 127 * np.abs(d16 - d) + 1e-6 * d
            assert (np.abs(deq.reshape(-1, 32) - blk) <= bound).all()
        else:
            assert o.tensor_type == t.tensor_type
            assert np.array_equal(np.asarray(o.data), np.asarray(t.data))
    # Every gwp linear weight except the 2x2 patch kernel is Q8_0.
    lin = [t.name for t in rs.tensors if t.name.startswith("gwp.") and t.name.endswith(".weight")
           and not t.name.endswith((".qn.weight", ".kn.weight", "ca_norm.weight"))]
    assert n_q8 == len(lin) - 1


def test_converted_metadata_and_inspection(converted):
    from wam_b200 import artifact

    src, dst, stats = converted
    rep = artifact.inspect(dst, artifact.Q8_POLICY_ID)
    assert rep["policy"] == artifact.Q8_POLICY_ID
    assert rep["components"]["gwp"]["q8_tensors"] > 0
    assert rep["components"]["gwp"]["stored_bytes"] == stats["gwp"]["stored_bytes"]
    assert stats["gwp"]["stored_bytes"] < stats["gwp"]["source_bytes"]
    rd = gguf.GGUFReader(str(dst))
    assert rd.get_field("gwp05.weight_policy").contents() == artifact.Q8_POLICY_ID
    assert rd.get_field("gwp05.conversion_policy").contents() == artifact.Q8_POLICY_ID
    # Geometry keys are carried over unchanged.
    rs = gguf.GGUFReader(str(src))
    for k in ("gwp05.hidden", "gwp05.n_layers", "gwp05.norm_eps", "gwp05.prompt_tokens"):
        assert rd.get_field(k).contents() == rs.get_field(k).contents()
    assert artifact.inspect(src, artifact.BF16_POLICY_ID)["policy"] == artifact.BF16_POLICY_ID


def test_converter_matches_fixture_quantiser(converted, tmp_path):
    """Tensors both writers quantise (rows = GGUF ne[0]) are byte-identical."""
    from oracle import synth
    from wam_b200 import artifact

    _, dst, _ = converted
    ref = tmp_path / "fixture_q8.gguf"
    write_artifact(ref, synth.TINY, q8=True)
    a = {t.name: t for t in gguf.GGUFReader(str(dst)).tensors}
    same = 0
    for t in gguf.GGUFReader(str(ref)).tensors:
        o = a[t.name]
        if o.tensor_type == t.tensor_type == gguf.GGMLQuantizationType.Q8_0 and \
           list(o.shape) == list(t.shape):
            assert np.array_equal(np.asarray(o.data), np.asarray(t.data)), t.name
            same += 1
    assert same > 20
    assert artifact.inspect(ref)["policy"] == "unlabelled"


@pytest.mark.parametrize("q8,policy", [(False, "mot-q8_0-v1"), (True, "mot-vae-bf16-qkv-v1")])
def test_inspect_rejects_policy_violations(tmp_path, q8, policy):
    from oracle import synth
    from wam_b200 import artifact

    p = tmp_path / "bad.gguf"
    write_artifact(p, synth.TINY, q8=q8, policy=policy)
    with pytest.raises(artifact.ContractError, match="dtype"):
        artifact.inspect(p)


def test_cli_convert_and_refuse_overwrite(converted, tmp_path, capsys):
    from wam_b200 import artifact

    src, _, _ = converted
    out = tmp_path / "cli.gguf"
    assert artifact.main(["convert", str(src), str(out)]) == 0
    assert '"valid": true' in capsys.readouterr().out
    assert artifact.main(["convert", str(src), str(out)]) == 1
    assert "refusing to overwrite" in capsys.readouterr().out
    assert artifact.main(["inspect", str(out), "--expect-policy", "mot-q8_0-v1"]) == 0
    assert artifact.main(["inspect", str(src), "--expect-policy", "mot-q8_0-v1"]) == 1
