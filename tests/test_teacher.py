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


def _split_forward(runner, ids, cuts):
    runner.reset()
    outs, start = [], 0
    for stop in (*cuts, ids.shape[1]):
        outs.append(runner.forward(ids[:, start:stop]))
        start = stop
    return torch.cat(outs, 1)


@pytest.mark.parametrize("cuts", [(3,), (2, 9), (1, 5, 6)])
def test_runner_chunks_match_one_pass_before_and_after_replacement(cuts):
    """The runner's cache carries attention KV, GDN conv windows and delta-rule states (and, once installed,
    TimeMix states) so that any split of a sequence gives the one-pass hidden states."""
    torch.manual_seed(len(cuts))
    model = tiny_model(seed=len(cuts))
    runner = Runner(model)
    ids = torch.randint(0, 64, (2, 12))
    runner.reset()
    one_pass = runner.forward(ids)
    torch.testing.assert_close(_split_forward(runner, ids, cuts), one_pass, atol=.03, rtol=.03)
    for layer in migration_order(model, expected=2):
        install(model, layer, {"head_size": 8, "backend": "reference"})
    runner.reset()
    replaced = runner.forward(ids)
    torch.testing.assert_close(_split_forward(runner, ids, cuts), replaced, atol=.03, rtol=.03)
    assert runner.cache.cursor == ids.shape[1]


def test_forward_through_layer_captures_the_same_boundary():
    """A forward that stops after the last migrated block captures what a full forward captures at that block,
    chunk after chunk, and advances the cache cursor the same way."""
    reference_model, short_model = tiny_model(seed=3), tiny_model(seed=3)
    runners = Runner(reference_model), Runner(short_model)
    captures = [Capture(m.model.layers[1].self_attn) for m in (reference_model, short_model)]
    try:
        for length in (5, 1, 4):
            ids = torch.randint(0, 64, (1, length))
            runners[0].forward(ids)
            runners[1].forward(ids, through_layer=1)
            for attr in ("x", "y"):
                torch.testing.assert_close(getattr(captures[1], attr), getattr(captures[0], attr),
                                           atol=.001, rtol=.001)
        assert runners[0].cache.cursor == runners[1].cache.cursor == 10
    finally:
        for capture in captures:
            capture.close()


def test_trainable_adapter_keeps_gradients_in_its_layer():
    """Only the installed TimeMix of the trained layer receives gradients from its distillation loss; the rest
    of the (frozen) model stays gradient-free."""
    teacher, student = tiny_model(seed=4), tiny_model(seed=4)
    teacher_runner, student_runner = Runner(teacher), Runner(student)
    adapter = install(student, 1, {"head_size": 8, "backend": "reference"}, trainable=True)
    adapter.__dict__["train_call"] = adapter.core
    capture = Capture(teacher.model.layers[1].self_attn)
    try:
        ids = torch.randint(0, 64, (1, 7))
        teacher_runner.forward(ids)
        adapter.teacher_input, adapter.debug_input = capture.x, True
        student_runner.forward(ids)
        loss = (adapter.prediction.float() - capture.y.float()).abs().mean()
        loss.backward()
        with_grad = {name for name, p in student.named_parameters() if p.grad is not None}
        assert with_grad
        assert all(name.startswith("model.layers.1.self_attn.core.") for name in with_grad)
    finally:
        capture.close()


def test_runner_state_dict_replays_the_same_continuation():
    """Saving the runner state after a prefix and loading it back reproduces the continuation exactly."""
    model = tiny_model(seed=5)
    install(model, 3, {"head_size": 8, "backend": "reference"})
    runner = Runner(model)
    runner.forward(torch.randint(0, 64, (1, 6)))
    saved = cpu_tree(runner.state_dict())
    tail = torch.randint(0, 64, (1, 4))
    first = runner.forward(tail)
    runner.forward(torch.randint(0, 64, (1, 2)))  # moves the cache on
    runner.load_state_dict(saved)
    torch.testing.assert_close(runner.forward(tail), first)


def test_isolated_state_is_invisible_to_the_training_stream():
    """Validation forwards inside ``isolated_state`` (other tokens, other lengths) leave the training cache where
    it was."""
    model = tiny_model(seed=6)
    install(model, 1, {"head_size": 8, "backend": "reference"})
    runner = Runner(model)
    prefix, nxt = torch.randint(0, 64, (1, 4)), torch.randint(0, 64, (1, 3))
    runner.forward(prefix)
    saved = cpu_tree(runner.state_dict())
    with isolated_state(runner):
        for length in (2, 5):
            runner.forward(torch.randint(0, 64, (1, length)))
    assert runner.cache.cursor == 4
    after = runner.forward(nxt)
    runner.load_state_dict(saved)
    torch.testing.assert_close(after, runner.forward(nxt))


def test_migration_order():
    model = tiny_model(depth=6)
    assert migration_order(model, expected=3) == [1, 3, 5]
    with pytest.raises(ValueError):
        migration_order(model, expected=2)
