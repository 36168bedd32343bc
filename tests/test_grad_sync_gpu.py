"""Peer-memory gradient exchange (reduce-scatter + clip + sharded AdamW + all-gather) on 2+ GPUs.

The pytest entry points launch this file under torchrun (one process per GPU, NVLS off) and check its
exit status; the worker compares the peer path with the NCCL all-reduce + full-update path and with a
host fp64 reference, and checks that an exchange whose peer never arrives ends with a status (no hang).
"""
import os
import socket
import subprocess
import sys
import types
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
pytestmark = [pytest.mark.gpu, pytest.mark.multi_gpu]
need2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                           reason="needs two GPUs")


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ranks():
    """Ranks per test: THESEUS_TEST_RANKS (up to the visible GPUs), else 2."""
    want = int(os.environ.get("THESEUS_TEST_RANKS", "2"))
    return max(2, min(want, torch.cuda.device_count()))


def _launch(mode, nproc=None):
    nproc = nproc or _ranks()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=str(ROOT))
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1", f"--master-port={_port()}", __file__, mode]
    out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    failed = "\n".join(line for line in out.stdout.splitlines() if line.startswith("RANK_FAILED"))
    assert out.returncode == 0, failed + "\n" + out.stdout[-3000:] + out.stderr[-3000:]
    return out.stdout


@need2
def test_peer_exchange_matches_nccl_path():
    assert "EXCHANGE_OK" in _launch("match")


@need2
def test_peer_exchange_odd_sizes_against_host_reference():
    assert "ODD_OK" in _launch("odd")


@need2
def test_missing_peer_times_out_with_status():
    assert "TIMEOUT_OK" in _launch("timeout")


# ---------------------------------------------------------------- worker (runs under torchrun)
def _student(topo, grad_sync, weights=None):
    from rwkv_theseus_b200.config import DEFAULTS
    from rwkv_theseus_b200.stage import Student
    cfg = DEFAULTS | {"head_size": 64, "backend": "cuda", "lr": 1e-3, "warmup_steps": 0, "clip_norm": 0.5,
                      "grad_sync": grad_sync}
    torch.manual_seed(0)
    return Student(types.SimpleNamespace(hidden_size=256, num_hidden_layers=8), 3, cfg, topo, weights=weights,
                   total_steps=10)


def _close_params(peer, nccl, steps, label, lr=1e-3):
    """Peer exchange against the NCCL all-reduce path. The two sum the ranks' gradients in different orders, so
    with more than two ranks an element whose gradients nearly cancel can take a different Adam step (its
    normalised moment m / sqrt(v) depends on the rounding of a tiny sum). Every element is within the largest
    possible drift (2 lr per update: each Adam step is below lr in size) and almost all (99.9%) within fp32
    rounding of each other; with two ranks the sums are identical and so is every element."""
    diff = (peer - nccl).abs()
    tight = diff <= 1e-7 + 1e-5 * nccl.abs()
    assert diff.max().item() <= 2 * lr * steps, (label, diff.max().item())
    assert tight.float().mean().item() >= 0.999, (label, 1 - tight.float().mean().item())
    if torch.distributed.get_world_size() <= 2:
        assert bool(tight.all()), (label, diff.max().item())


def _match(topo):
    dev = topo.device
    peer = _student(topo, "peer")
    nccl = _student(topo, "nccl", weights={k: v.detach().clone() for k, v in peer.core.state_dict().items()})
    assert torch.equal(peer.flat.param, nccl.flat.param)
    n = peer.flat.numel
    for step in range(4):
        g = torch.Generator(device=dev).manual_seed(1000 + 17 * step + topo.rank)
        grad = torch.randn(n, device=dev, generator=g) * (0.01 if step % 2 else 3.0)  # clipped / unclipped
        stats = torch.tensor([1.5 + topo.rank, 0.25, 64.0 + 8 * topo.rank], device=dev)

        for s in (peer, nccl):
            s.flat.grad.copy_(grad)
            s.grads_live = True  # injected gradients stand for this update's micro-steps
            s.stats.copy_(stats)
            s.reduce()
            s.update()
        topo.join_grad_sync()
        torch.cuda.synchronize()
        if step == 2:
            try:
                peer.weights()
            except RuntimeError as err:
                assert "sync_state" in str(err)
            else:
                raise AssertionError("sharded weights must not be readable")
        assert torch.equal(peer.fused.shadow, nccl.fused.shadow) or \
            (peer.fused.shadow.float() - nccl.fused.shadow.float()).abs().max() <= 1e-2 * nccl.flat.param.abs().max()
        tail = slice(peer.decay_numel, None)  # fp32 non-decay parameters are gathered every update
        _close_params(peer.flat.param[tail], nccl.flat.param[tail], step + 1, f"non-decay step {step}")
        if step == 1:
            peer.sync_state()  # gather the sharded fp32 masters and moments mid-run; training continues
            torch.cuda.synchronize()
            _close_params(peer.flat.param, nccl.flat.param, step + 1, f"all parameters step {step}")
        assert torch.equal(peer.fused.shadow, peer.flat.param.to(torch.bfloat16)) or step != 1, step
        assert torch.allclose(peer.report, nccl.report, rtol=1e-5), (step, peer.report, nccl.report)
        assert not peer.stats.any(), step
    topo.check_grad_sync()
    peer.sync_state()
    torch.cuda.synchronize()
    _close_params(peer.flat.param, nccl.flat.param, 4, "all parameters, end")
    assert torch.equal(peer.fused.shadow, peer.flat.param.to(torch.bfloat16))
    for name, atol in (("exp_avg", 1e-9), ("exp_avg_sq", 1e-12)):  # moments: same rule as the parameters
        mine, theirs = getattr(peer.flat, name), getattr(nccl.flat, name)
        diff = (mine - theirs).abs()
        tight = diff <= atol + 1e-5 * theirs.abs()
        assert diff.max().item() <= 1e-3 * theirs.abs().max().item(), (name, diff.max().item())
        assert tight.float().mean().item() >= 0.999 and (topo.world > 2 or bool(tight.all())), name
    everyone = [torch.empty_like(peer.flat.param) for _ in range(topo.world)]
    torch.distributed.all_gather(everyone, peer.flat.param, group=topo.student_group)
    assert all(torch.equal(everyone[0], e) for e in everyone)
    print("EXCHANGE_OK", flush=True)


def _fake(topo, n, decay):
    dev = topo.device
    flat = types.SimpleNamespace(numel=n, param=torch.zeros(n, device=dev), grad=torch.zeros(n, device=dev),
                                 exp_avg=torch.zeros(n, device=dev), exp_avg_sq=torch.zeros(n, device=dev))
    return types.SimpleNamespace(flat=flat, fused=types.SimpleNamespace(shadow=torch.zeros(n, device=dev,
                                                                                          dtype=torch.bfloat16)),
                                 stats=torch.zeros(3, device=dev), report=torch.zeros(5, device=dev),
                                 decay_numel=decay,
                                 cfg={"betas": [0.9, 0.999], "adam_eps": 1e-8, "weight_decay": 0.1, "clip_norm": 1.0})


def _odd(topo):
    from rwkv_theseus_b200.parallel.grad_sync import PeerGradExchange
    dev = topo.device
    ex = PeerGradExchange(topo, blocks=3, limit_s=30.0)
    for n, decay in ((1001, 500), (7, 3), (4096 + 2, 4096)):
        st = _fake(topo, n, decay)
        ex.register(st)
        g0 = torch.Generator(device=dev).manual_seed(5)
        p0 = torch.randn(n, device=dev, generator=g0)
        st.flat.param.copy_(p0)
        p = p0.double().cpu()
        m = torch.zeros(n, dtype=torch.float64)
        v = torch.zeros(n, dtype=torch.float64)
        for step in range(1, 3):
            grads = []
            for q in range(topo.world):
                gq = torch.Generator(device=dev).manual_seed(77 * step + q)
                grads.append(torch.randn(n, device=dev, generator=gq) * 2)
            st.flat.grad.copy_(grads[topo.rank])
            st.stats.copy_(torch.tensor([1.0, 2.0, 10.0], device=dev))
            ex.update(st, 1e-2, step)
            ex.gather_state(st)
            torch.cuda.synchronize()
            count = 10.0 * topo.world
            gsum = sum(x.double().cpu() for x in grads) / count
            norm = gsum.norm().item()
            gsum = gsum * min(1.0, 1.0 / (norm + 1e-6))
            p[:decay] *= 1 - 1e-2 * 0.1
            m = m + 0.1 * (gsum - m)
            v = 0.999 * v + 0.001 * gsum * gsum
            p = p - (1e-2 / (1 - 0.9 ** step)) * m / (v.sqrt() / (1 - 0.999 ** step) ** 0.5 + 1e-8)
            assert torch.allclose(st.flat.param.double().cpu(), p, rtol=1e-4, atol=1e-6), (n, step)
            assert abs(st.report[3].item() - norm) <= 1e-4 * norm, (n, step)
            assert st.report[2].item() == count
    ex.check()
    ex.close()
    print("ODD_OK", flush=True)


def _timeout(topo):
    from rwkv_theseus_b200.parallel.grad_sync import PeerGradExchange
    ex = PeerGradExchange(topo, blocks=2, limit_s=1.0)
    st = _fake(topo, 64, 32)
    ex.register(st)  # collective mapping on both ranks; only the exchange itself is skipped by rank 1
    topo.barrier()
    if topo.rank == 0:  # rank 1 never joins this exchange: every wait of rank 0 runs out after 1 s
        ex.update(st, 1e-3, 1)
        ex.wait()
        torch.cuda.synchronize()
        try:
            ex.check()
        except RuntimeError as err:
            assert "timed out" in str(err)
        else:
            raise AssertionError("missing timeout status")
        assert torch.equal(st.flat.param, torch.zeros_like(st.flat.param))  # nothing applied
    topo.barrier()
    ex.close()
    print("TIMEOUT_OK", flush=True)


def main(mode):
    sys.path.insert(0, str(ROOT))
    from rwkv_theseus_b200.parallel.topology import Topology
    topo = Topology("nccl", timeout_minutes=2)
    try:
        {"match": _match, "odd": _odd, "timeout": _timeout}[mode](topo)
    except BaseException as err:  # one line per failing rank, which the launcher puts first in its report
        print(f"RANK_FAILED rank {topo.rank}: {type(err).__name__}: {err!r}"[:600], flush=True)
        raise
    finally:
        topo.close()


if __name__ == "__main__":
    main(sys.argv[1])
