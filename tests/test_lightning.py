"""Lightning PTH tools: HF hybrid -> PTH export and TimeMix splicing (the reference's
``tests/test_replace_timemix_lightning.py`` contract plus an export round trip on a tiny hybrid)."""
import json

import pytest
import torch
from safetensors.torch import save_file

from convert_qwen2rwkv_lightning import convert
from replace_timemix_lightning import BASE_FORMAT, OUTPUT_FORMAT, export_tensor, replace, sidecar
from rwkv_theseus_b200.models.hf_io import random_model, save_model
from rwkv_theseus_b200.models.qwen35 import HybridConfig
from rwkv_theseus_b200.models.timemix import TimeMix


def tiny_hybrid():
    return HybridConfig(vocab_size=300, hidden_size=128, intermediate_size=256, num_hidden_layers=4,
                        num_attention_heads=4, num_key_value_heads=2, head_dim=32, linear_num_key_heads=2,
                        linear_num_value_heads=4, linear_key_head_dim=32, linear_value_head_dim=32,
                        linear_conv_kernel_dim=4, layer_types=["linear_attention"] * 3 + ["full_attention"],
                        rope_theta=1e6, partial_rotary_factor=0.25)


def test_export_maps_every_tensor_and_splits_packed_rows(tmp_path):
    model = random_model(tiny_hybrid(), "cpu", dtype=torch.bfloat16, seed=3)
    save_model(model, tmp_path / "hf")
    out = tmp_path / "out" / "hybrid.pth"
    convert(tmp_path / "hf", out, verify=True, quiet=True)
    pth = torch.load(out, weights_only=True)
    sd = model.state_dict()
    kd, qd = 2 * 32, 4 * 32
    qkv = sd["model.layers.0.linear_attn.in_proj_qkv.weight"]
    assert pth["blocks.0.att.receptance.weight"].equal(qkv[:kd])
    assert pth["blocks.0.att.key.weight"].equal(qkv[kd:2 * kd])
    assert pth["blocks.0.att.value.weight"].equal(qkv[2 * kd:])
    q = sd["model.layers.3.self_attn.q_proj.weight"].view(4, 2, 32, 128)
    assert pth["blocks.3.att.receptance.weight"].equal(q[:, 0].reshape(qd, 128))
    assert pth["blocks.3.att.gate.weight"].equal(q[:, 1].reshape(qd, 128))
    assert pth["blocks.0.att.conv1d.weight"].shape == (2 * kd + 4 * 32, 4)
    assert pth["blocks.1.ffn.key.weight"].equal(sd["model.layers.1.mlp.up_proj.weight"])
    assert pth["head.weight"].equal(sd["lm_head.weight"]) and pth["emb.weight"].dtype == torch.bfloat16
    meta = json.loads(sidecar(out, "config").read_text())
    assert meta["format"] == BASE_FORMAT and meta["geometry"]["layer_types"][3] == "full_attention"
    assert meta["contract"]["gdn_state_layout"] == "B,Hv,K,V"
    manifest = json.loads(sidecar(out, "manifest").read_text())
    assert {e["target"] for e in manifest["tensors"]} == set(pth)
    with pytest.raises(FileExistsError):
        convert(tmp_path / "hf", out, quiet=True)


def test_export_rejects_unmapped_text_tensors(tmp_path):
    model = random_model(tiny_hybrid(), "cpu", seed=1)
    state = dict(model.state_dict())
    state["model.layers.0.linear_attn.mystery.weight"] = torch.zeros(2)
    save_model(model, tmp_path / "hf", extra_state=state)
    with pytest.raises(ValueError, match="Unmapped TEXT tensors"):
        convert(tmp_path / "hf", tmp_path / "x.pth", dry_run=True, quiet=True)


def _base(tmp_path, layer_types, tensors, hidden=128):
    base = tmp_path / "base.pth"
    torch.save(tensors, base)
    geometry = {"hidden_size": hidden, "num_hidden_layers": len(layer_types), "layer_types": layer_types,
                "linear_num_value_heads": 2, "linear_key_head_dim": 128, "linear_value_head_dim": 128}
    sidecar(base, "config").write_text(json.dumps({"format": BASE_FORMAT, "weights_file": base.name,
                                                   "geometry": geometry}))
    sidecar(base, "manifest").write_text(json.dumps({"format": BASE_FORMAT, "tensors": [
        {"target": k, "source": k} for k in tensors]}))
    return base


@pytest.mark.parametrize("head_size", [64, 128])
def test_splice_replaces_one_layer_with_the_latest_snapshot(tmp_path, head_size):
    original = {"emb.weight": torch.arange(256, dtype=torch.bfloat16).reshape(2, 128),
                "blocks.0.att.A_log": torch.arange(2, dtype=torch.bfloat16),
                "blocks.3.att.q_norm.weight": torch.ones(8, dtype=torch.bfloat16),
                "blocks.3.att.key.weight": torch.ones(8, 128, dtype=torch.bfloat16)}
    base = _base(tmp_path, ["linear_attention"] * 3 + ["full_attention"], original)
    snaps = tmp_path / "weights"
    snaps.mkdir()
    core = TimeMix(128, 3, 4, head_size=head_size, backend="reference")
    state = {"3." + k: v.detach().float().contiguous() for k, v in core.state_dict().items()}
    save_file(state, snaps / "stage_1.safetensors")
    newer = {"3.x_r": torch.full_like(state["3.x_r"], 0.375)}
    save_file(newer, snaps / "stage_10.safetensors")  # natural order: stage_10 after stage_1
    out = tmp_path / "replaced.pth"
    replace(base, snaps, out, [3], verify=True, quiet=True)
    got = torch.load(out, weights_only=True)
    assert got["blocks.0.att.A_log"].equal(original["blocks.0.att.A_log"])
    assert "blocks.3.att.q_norm.weight" not in got and "blocks.3.att.key.weight" in got
    assert got["blocks.3.att.x_r"].equal(newer["3.x_r"].to(torch.bfloat16).reshape(-1))
    assert len([k for k in got if k.startswith("blocks.3.att.")]) == len(state)
    for key, value in state.items():
        if key != "3.x_r":
            assert got["blocks.3.att." + key[2:]].equal(export_tensor(key[2:], value.to(torch.bfloat16)))
    meta = json.loads(sidecar(out, "config").read_text())
    assert meta["format"] == OUTPUT_FORMAT and meta["requires_hybrid_backend"] is True
    assert meta["contract"]["timemix_weight_layout"] == "out_in_row_major_vectors_flat_v1"
    assert meta["geometry"]["layer_types"][3] == "rwkv7_timemix"
    assert meta["wkv_layers"]["3"]["head_size"] == head_size
    entries = json.loads(sidecar(out, "manifest").read_text())["tensors"]
    assert next(e for e in entries if e["target"] == "blocks.3.att.x_r")["file"] == "stage_10.safetensors"
    with pytest.raises(ValueError, match="was trained with head_size"):
        replace(base, snaps, out, [3], head_size=128 if head_size == 64 else 64, dry_run=True)
    second = tmp_path / "second.pth"  # incremental: splice again into the spliced file, keep source dtype
    replace(out, snaps / "stage_1.safetensors", second, [3], head_size=head_size, dtype="source", verify=True,
            quiet=True)
    got2 = torch.load(second, weights_only=True)
    assert got2["blocks.3.att.w1"].dtype == torch.float32 and got2["blocks.3.att.w1"].equal(state["3.w1"].T)
    for layers in ([], [-1], [3, 3]):
        with pytest.raises(ValueError, match="distinct nonnegative"):
            replace(base, snaps, second, layers, dry_run=True)


def test_splice_rejects_an_incomplete_layer(tmp_path):
    base = _base(tmp_path, ["linear_attention"] * 3 + ["full_attention"],
                 {"emb.weight": torch.zeros(2, 128), "blocks.3.att.key.weight": torch.zeros(8, 128)})
    snaps = tmp_path / "weights"
    snaps.mkdir()
    save_file({"3.x_r": torch.zeros(1, 1, 128)}, snaps / "partial.safetensors")
    with pytest.raises(ValueError, match="incomplete"):
        replace(base, snaps, tmp_path / "out.pth", [3], head_size=64, dry_run=True)


def test_export_layout_of_every_timemix_parameter():
    core = TimeMix(64, 0, 2, head_size=64, backend="reference")
    for name, value in core.state_dict().items():
        out = export_tensor(name, value)
        if name in {"w1", "w2", "a1", "a2", "g1", "g2"}:
            assert out.equal(value.T)
        elif value.ndim == 3:
            assert out.shape == (64,)
        else:
            assert out.equal(value)
        assert out.is_contiguous()


def test_splice_infers_mixed_head_sizes(tmp_path):
    base = _base(tmp_path, ["full_attention", "full_attention"],
                 {"emb.weight": torch.zeros(2, 128), "blocks.0.att.q_norm.weight": torch.ones(64),
                  "blocks.1.att.q_norm.weight": torch.ones(64)})
    tensors = {}
    for layer, size in enumerate((64, 128)):
        core = TimeMix(128, layer, 2, head_size=size, backend="reference")
        tensors.update({f"{layer}.{k}": v.detach().contiguous() for k, v in core.state_dict().items()})
    src = tmp_path / "migrated.safetensors"
    save_file(tensors, src)
    out = tmp_path / "out.pth"
    replace(base, src, out, [0, 1], verify=True, quiet=True)
    got = torch.load(out, weights_only=True)
    assert got["blocks.0.att.r_k"].shape == (2, 64) and got["blocks.1.att.r_k"].shape == (1, 128)
    meta = json.loads(sidecar(out, "config").read_text())
    assert meta["wkv_layers"]["0"]["head_size"] == 64 and meta["wkv_layers"]["1"]["head_size"] == 128
