"""Own hybrid teacher vs the HF Qwen3.5 implementation (oracle) and runner behaviour."""
import pytest
import torch

from fixtures import save_tiny, tiny_model
from rwkv_theseus_b200.checkpoint import cpu_tree
from rwkv_theseus_b200.models.hf_io import load_model
from rwkv_theseus_b200.models.qwen35 import HybridCache
from rwkv_theseus_b200.models.runner import Capture, Runner, install, isolated_state, migration_order


def _hf_tiny(tmp_path, value_heads=4):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.Qwen3_5TextConfig(
        hidden_size=32, intermediate_size=64, num_hidden_layers=4, num_attention_heads=2, num_key_value_heads=1,
        head_dim=16, vocab_size=64, layer_types=["linear_attention", "full_attention"] * 2,
        linear_num_key_heads=2, linear_num_value_heads=value_heads, linear_key_head_dim=8,
        linear_value_head_dim=8, linear_conv_kernel_dim=4,
        rope_parameters={"rope_type": "default", "rope_theta": 10000., "partial_rotary_factor": .5,
                         "mrope_section": [1, 1, 0]})
    cfg._attn_implementation = "sdpa"
    hf = transformers.Qwen3_5ForCausalLM(cfg).float().eval()
    with torch.no_grad():
        for name, p in hf.named_parameters():
            if "norm" in name and "linear_attn" not in name:
                p.normal_(0, 0.1)
    hf.save_pretrained(tmp_path / "hf")
    return hf, tmp_path / "hf"


def test_matches_hf_one_shot_and_carries_state_across_chunks(tmp_path):
    hf, path = _hf_tiny(tmp_path)
    mine = load_model(path, "cpu", dtype=torch.float32)
    ids = torch.randint(0, 64, (2, 13))
    with torch.no_grad():
        expected = hf.model(input_ids=ids).last_hidden_state
        full = mine.model(ids, torch.arange(13), HybridCache(mine.config))
        cache, parts = HybridCache(mine.config), []
        for a, b in [(0, 4), (4, 5), (5, 13)]:
            parts.append(mine.model(ids[:, a:b], torch.arange(a, b), cache))
            cache.cursor = b
        logits = mine.lm_head(full)
    torch.testing.assert_close(full, expected, atol=2e-5, rtol=1e-4)
    torch.testing.assert_close(torch.cat(parts, 1), expected, atol=2e-5, rtol=1e-4)
    torch.testing.assert_close(logits, hf.lm_head(expected), atol=2e-5, rtol=1e-4)


def test_hf_layout_roundtrip_and_strict_loader(tmp_path):
    model = tiny_model()
    save_tiny(tmp_path / "m")
    loaded = load_model(tmp_path / "m", "cpu")
    for (n, a), (m, b) in zip(model.state_dict().items(), loaded.state_dict().items()):
        assert n == m
        torch.testing.assert_close(a, b)


def test_cached_chunks_and_all_replaced():
    model = tiny_model()
    runner = Runner(model)
    ids = torch.randint(0, 64, (1, 11))
    full = runner.forward(ids)
    runner.reset()
    parts = [runner.forward(ids[:, :4]), runner.forward(ids[:, 4:7]), runner.forward(ids[:, 7:])]
    torch.testing.assert_close(torch.cat(parts, 1), full, atol=.03, rtol=.03)
    for layer in [3, 1]:
        install(model, layer, {"head_size": 8, "backend": "reference"})
    runner.reset()
    full = runner.forward(ids)
    runner.reset()
    pieces = [runner.forward(ids[:, :4]), runner.forward(ids[:, 4:])]
    torch.testing.assert_close(torch.cat(pieces, 1), full, atol=.03, rtol=.03)
    assert runner.cache.cursor == 11


def test_truncated_teacher_matches_full_boundary_across_chunks():
    full_model, short_model = tiny_model(), tiny_model()
    full_runner, short_runner = Runner(full_model), Runner(short_model)
    full_capture = Capture(full_model.model.layers[1].self_attn)
    short_capture = Capture(short_model.model.layers[1].self_attn)
    try:
        for ids in (torch.randint(0, 64, (1, 6)), torch.randint(0, 64, (1, 3))):
            full_runner.forward(ids)
            short_runner.forward(ids, through_layer=1)
            torch.testing.assert_close(short_capture.x, full_capture.x, atol=.001, rtol=.001)
            torch.testing.assert_close(short_capture.y, full_capture.y, atol=.001, rtol=.001)
        assert full_runner.cache.cursor == short_runner.cache.cursor == 9
    finally:
        full_capture.close()
        short_capture.close()


def test_adapter_only_current_layer_has_grad_and_runner_restore():
    teacher, student = tiny_model(), tiny_model()
    tr, sr = Runner(teacher), Runner(student)
    adapter = install(student, 3, {"head_size": 8, "backend": "reference"}, trainable=True)
    adapter.__dict__["train_call"] = adapter.core
    capture = Capture(teacher.model.layers[3].self_attn)
    ids = torch.randint(0, 64, (1, 6))
    tr.forward(ids)
    adapter.teacher_input = capture.x
    adapter.debug_input = True
    sr.forward(ids)
    (adapter.prediction.float() - capture.y.float()).square().mean().backward()
    grads = [n for n, p in student.named_parameters() if p.grad is not None]
    assert grads and all(n.startswith("model.layers.3.self_attn.core.") for n in grads)
    adapter.teacher_input = adapter.prediction = None
    state = cpu_tree(sr.state_dict())
    more = torch.randint(0, 64, (1, 3))
    expected = sr.forward(more)
    sr.load_state_dict(state)
    torch.testing.assert_close(sr.forward(more), expected, atol=.001, rtol=.001)
    capture.close()


def test_isolated_validation_does_not_change_training():
    model = tiny_model()
    install(model, 3, {"head_size": 8, "backend": "reference"})
    runner = Runner(model)
    ids = torch.randint(0, 64, (1, 5))
    runner.forward(ids)
    state = cpu_tree(runner.state_dict())
    with isolated_state(runner):
        runner.forward(ids)
        runner.forward(ids)
    actual = runner.forward(ids)
    runner.load_state_dict(state)
    torch.testing.assert_close(actual, runner.forward(ids))


def test_migration_order():
    model = tiny_model(depth=6)
    assert migration_order(model, expected=3) == [1, 3, 5]
    with pytest.raises(ValueError):
        migration_order(model, expected=2)
