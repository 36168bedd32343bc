"""Multi-process workers for tests/test_distributed.py (launched with torch.distributed.run, Gloo, CPU)."""
import sys
import types
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from rwkv_theseus_b200.config import DEFAULTS  # noqa: E402
from rwkv_theseus_b200.losses import loss_sum, statistics  # noqa: E402
from rwkv_theseus_b200.models.timemix import TimeMix  # noqa: E402
from rwkv_theseus_b200.parallel.topology import Topology  # noqa: E402
from rwkv_theseus_b200.stage import Student  # noqa: E402


def weighted():
    """Rank-dependent sequence lengths: the reduced, count-divided gradient equals the serial one."""
    torch.set_num_threads(1)
    topo = Topology("gloo")
    cfg = DEFAULTS | {"head_size": 4, "backend": "reference", "lora_rank": 8, "gate_lora_rank": 8}
    torch.manual_seed(111)
    student = Student(types.SimpleNamespace(hidden_size=16, num_hidden_layers=4), 1, cfg, topo)
    with torch.no_grad():
        student.core.output.weight.normal_(0, 0.01)
    serial = TimeMix(16, 1, 4, 4, "reference", lora_rank=8, gate_lora_rank=8)
    serial.load_state_dict(student.core.state_dict())
    torch.manual_seed(222)
    data = [(torch.randn(1, n, 16), torch.randn(1, n, 16)) for n in range(3, 3 + topo.world)]
    x, target = data[topo.rank]
    total = 0.0
    for xs, ts in data:  # same bf16 autocast as the student's micro-step
        with torch.autocast("cpu", dtype=torch.bfloat16):
            y, _ = serial(xs)
        total = total + loss_sum(statistics(y, ts), 0.0)
    total.backward()  # unscaled: bf16 autocast backward is not invariant to a scaled loss
    student.micro_step(x, target)
    student.reduce()
    count = student.stats[2].item()
    assert count == sum(range(3, 3 + topo.world))
    for (name, p), q in zip(student.core.named_parameters(), serial.parameters()):
        torch.testing.assert_close(p.grad / count, q.grad / count, atol=1e-7, rtol=1e-5, msg=name)
    topo.barrier()
    dist.destroy_process_group()


def mismatch():
    """Ranks that disagree on the run configuration are rejected before any collective schedule."""
    topo = Topology("gloo")
    try:
        topo.assert_same({"grad_accum_steps": topo.rank + 1}, "test config")
    except ValueError as err:
        assert "Ranks disagree" in str(err)
    else:
        raise AssertionError("an inconsistent configuration was accepted")
    topo.close()


def failing():
    """Rank 1 dies before a collective; rank 0's all-reduce must end with an error (short PG timeout)."""
    topo = Topology("gloo", timeout_minutes=0.15)
    if topo.rank == 1:
        raise RuntimeError("injected failure on rank 1")
    x = torch.ones(4)
    dist.all_reduce(x, group=topo.student_group)  # never completes normally: rank 1 is gone
    raise AssertionError("all-reduce with a dead peer returned")


if __name__ == "__main__":
    {"weighted": weighted, "mismatch": mismatch, "failing": failing}[sys.argv[1]]()
