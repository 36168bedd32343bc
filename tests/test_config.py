"""This implementation's config keys: defaults, strict typing and their place among the keys a resume may change."""
import pytest

from rwkv_theseus_b200.checkpoint import MUTABLE_KEYS
from rwkv_theseus_b200.config import DEFAULTS, make_config

OWN_KEYS = {"lora_rank": None, "gate_lora_rank": None, "fused_optimizer": True, "grad_sync": "peer",
            "student_graphs": True, "overlap_students": True}


def test_own_keys_have_their_defaults():
    cfg = make_config({})
    for key, default in OWN_KEYS.items():
        assert DEFAULTS[key] == default and cfg[key] == default, key


@pytest.mark.parametrize("override", [{"overlap_students": "yes"}, {"overlap_students": 1},
                                      {"student_graphs": 0}, {"grad_sync": "ring"}, {"fused_optimizer": None}])
def test_own_keys_are_strictly_typed(override):
    with pytest.raises(ValueError):
        make_config(override)


def test_schedule_keys_may_change_on_resume():
    """Stream and graph scheduling do not change what is computed, so a resumed run may switch them."""
    for key in ("overlap_students", "student_graphs", "grad_sync", "fused_optimizer"):
        assert key in MUTABLE_KEYS
    assert make_config({"overlap_students": False})["overlap_students"] is False
