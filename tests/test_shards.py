"""NF24 shard directories (triposplat_nf24_i16_v1): the loader reads shards written by the
reference's own packer (tests/golden/shards_ref, made by tests/golden/make_golden.py from
tests/golden/shards_src.safetensors), its codes equal this repo's packer on the same source
weights, corruption is caught by the sha256 check, and shards written here have the
reference's manifest structure and load back unchanged.  CPU only (device "cpu")."""
import json
import shutil
from pathlib import Path

import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def _source():
    from safetensors.torch import load_file

    return load_file((GOLDEN / "shards_src.safetensors").as_posix())


def test_reference_shards_load_and_match_this_packer():
    from nf24_pack import quantize_nf24_i16_per_output_channel
    from nf24_shards import load_nf24_shards

    src = _source()
    sh = load_nf24_shards(GOLDEN / "shards_ref", device="cpu", verify_checksums=True)
    assert set(sh.linears) == {"blocks.0.attn.qkv", "blocks.0.mlp.fc1", "head"}
    for name, lin in sh.linears.items():
        codes, scales, _ = quantize_nf24_i16_per_output_channel(src[name + ".weight"])
        assert torch.equal(lin.code01, codes[0]) and torch.equal(lin.q2, codes[1])
        assert torch.equal(lin.scale, scales[0])
        bias = src.get(name + ".bias", torch.zeros(lin.code01.shape[1]))
        assert torch.equal(lin.bias, bias)
        assert lin.has_bias == (name + ".bias" in src)
    assert set(sh.non_linear) == {"blocks.0.norm.gamma", "pos_table"}
    for k, v in sh.non_linear.items():
        assert torch.equal(v, src[k])
    assert sh.checksums_verified and sh.loaded_bytes == sh.manifest["packed_bytes"]


def test_checksum_mismatch_and_bad_manifest(tmp_path):
    from nf24_shards import load_nf24_shards

    d = tmp_path / "shards"
    shutil.copytree(GOLDEN / "shards_ref", d)
    m = json.loads((d / "manifest.json").read_text())
    f = d / m["linears"]["head"]["file"]
    raw = bytearray(f.read_bytes())
    raw[-1] ^= 0x01  # flip one bit of the last code byte
    f.write_bytes(bytes(raw))
    with pytest.raises(RuntimeError, match="checksum"):
        load_nf24_shards(d, device="cpu", verify_checksums=True)
    load_nf24_shards(d, device="cpu")  # unverified load still reads it
    m["format"] = "other"
    (d / "manifest.json").write_text(json.dumps(m))
    with pytest.raises(RuntimeError, match="invalid"):
        load_nf24_shards(d, device="cpu")


def test_written_shards_round_trip_with_reference_manifest_layout(tmp_path):
    from nf24_shards import load_nf24_shards, save_nf24_shards

    ref = load_nf24_shards(GOLDEN / "shards_ref", device="cpu")
    man = save_nf24_shards(ref.linears, tmp_path / "out", non_linear=ref.non_linear,
                           source=ref.manifest["source"],
                           has_bias={n: lin.has_bias for n, lin in ref.linears.items()})
    ref_man = ref.manifest
    assert set(man) == set(ref_man)
    for name in ref_man["linears"]:
        assert set(man["linears"][name]) == set(ref_man["linears"][name])
        assert man["linears"][name]["file"] == ref_man["linears"][name]["file"]
        for key in ("in_features", "out_features", "has_bias", "weight_elements"):
            assert man["linears"][name][key] == ref_man["linears"][name][key]
    back = load_nf24_shards(tmp_path / "out", device="cpu", verify_checksums=True)
    for name, lin in ref.linears.items():
        for a in ("code01", "q2", "scale", "bias"):
            assert torch.equal(getattr(back.linears[name], a), getattr(lin, a))
    for k, v in ref.non_linear.items():
        assert torch.equal(back.non_linear[k], v)


def test_flow_weights_shard_round_trip_cpu(tmp_path):
    """The synthetic model's weights go through a shard directory unchanged (CPU)."""
    from flow_model import FlowSpec, make_weights
    from nf24_shards import load_flow_weights, save_flow_weights

    spec = FlowSpec.small(blocks=1)
    w = make_weights(spec, seed=3, device="cpu")
    save_flow_weights(w, tmp_path / "m")
    w2 = load_flow_weights(tmp_path / "m", spec, device="cpu", verify_checksums=True)
    for name, lin in w.linears.items():
        for a in ("code01", "q2", "scale", "bias"):
            assert torch.equal(getattr(w2.linears[name], a), getattr(lin, a))
    for k, v in w.params.items():
        assert torch.equal(w2.params[k], v)
