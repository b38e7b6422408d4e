"""Sequence-parallel prefill (`siso.siso_segment_seq_parallel`): each rank scans one
L-slice, and the exchange must reproduce the chained segments of ``siso.py:154-216``.

CPU: 2 and 4 gloo ranks, the scan itself stood in by the oracle's `siso_segment`
(injected as ``segment_fn``), so the angle offsets, the linear carry rebuild and the
seed bookkeeping are checked without a GPU.  GPU (needs 2 devices, skipped otherwise):
2 NCCL ranks on the CUDA kernels against one device scanning the whole sequence."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

B, H, L, N, P, NR, CHUNK = 2, 3, 256, 16, 16, 4, 32


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _case(seed=3):
    from oracle import siso_oracle as O
    from tests.inputs import make_inputs

    x = make_inputs(B, H, L, state_dim=N, headdim=P, n_angles=NR, seed=seed)
    x["dt_bias"] = torch.randn(H, generator=torch.Generator().manual_seed(seed), dtype=torch.float64) * 0.3
    g = torch.Generator().manual_seed(seed + 1)
    st = O.SISOState(ssm=torch.randn(B, H, P, N, generator=g, dtype=torch.float64) * 0.3,
                     k=torch.randn(B, H, N, generator=g, dtype=torch.float64),
                     v=torch.randn(B, H, P, generator=g, dtype=torch.float64),
                     phi=torch.rand(B, H, NR, generator=g, dtype=torch.float64) * 6.0)
    return x, st


def _args(x, lo, hi):
    sl = lambda t, ax: t.narrow(ax, lo, hi - lo)
    return (sl(x["q"], 1), sl(x["k"], 1), sl(x["v"], 2), sl(x["dt_raw"], 1), sl(x["a_raw"], 1),
            sl(x["trap_raw"], 1), sl(x["angles"], 1), x["dt_bias"], x["q_bias"], x["k_bias"], x["d_skip"],
            sl(x["z"], 2))


def _oracle_seg(*a, state=None, a_floor=1e-4, chunk=128, policy_name="f32"):
    from mamba3_b200.siso import SISOOutput
    from mamba3_b200.state import SISOState
    from oracle import siso_oracle as O

    st = None if state is None else O.SISOState(*(t.double() for t in state))
    y, fin = O.siso_segment(*(t.double() for t in a[:10]), d_skip=a[10].double(), z=a[11].double(), state=st,
                            a_floor=a_floor, chunk=chunk, policy="f32")
    return SISOOutput(y=y, state=SISOState(*fin))


def _worker(rank, world, port, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "mamba3-siso-tpu_b200")):
        sys.path.insert(0, p)
    from mamba3_b200.siso import siso_segment_seq_parallel
    from mamba3_b200.state import SISOState

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    x, st = _case()
    per = L // world
    out = siso_segment_seq_parallel(*_args(x, rank * per, (rank + 1) * per), state=SISOState(*st), chunk=CHUNK,
                                    policy_name="f32", segment_fn=_oracle_seg)
    q.put((rank, out.y.double().numpy(), [t.double().numpy() for t in out.state]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_seq_parallel_matches_chained_segments_gloo(world):
    from oracle import siso_oracle as O

    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, qu)) for r in range(world)]
    for p in procs:
        p.start()
    res = {r: (y, s) for r, y, s in (qu.get(timeout=300) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, st = _case()
    y_ref, fin = O.siso_segment(*_args(x, 0, L)[:10], d_skip=x["d_skip"], z=x["z"], state=st, chunk=CHUNK,
                                policy="f32")
    per = L // world
    for r in range(world):
        y, s = res[r]
        want = y_ref[:, :, r * per:(r + 1) * per]
        assert torch.allclose(torch.from_numpy(y), want, rtol=1e-5, atol=1e-5), f"rank {r} y"
        if r == world - 1:
            for name, a, b in zip(("ssm", "k", "v"), s[:3], fin[:3]):
                assert torch.allclose(torch.from_numpy(a), b, rtol=1e-5, atol=1e-5), name
            d = torch.remainder(torch.from_numpy(s[3]) - fin.phi + torch.pi, 2 * torch.pi) - torch.pi
            assert d.abs().max() < 1e-5


def _gpu_worker(rank, world, port, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "mamba3-siso-tpu_b200")):
        sys.path.insert(0, p)
    from mamba3_b200.siso import siso_segment, siso_segment_seq_parallel
    from mamba3_b200.state import SISOState

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    x, st = _gpu_case()
    dev = f"cuda:{rank}"
    xd = {k_: (t.to(dev, torch.bfloat16) if k_ in ("q", "k", "v", "z") else t.to(dev, torch.float32))
          for k_, t in x.items()}
    std = SISOState(*(t.to(dev, torch.float32) for t in st))
    per = GL // world
    out = siso_segment_seq_parallel(*_args(xd, rank * per, (rank + 1) * per), state=std, chunk=128,
                                    policy_name="bf16")
    res = [out.y.float().cpu().numpy()] + [t.cpu().numpy() for t in out.state]
    if rank == 0:  # the whole sequence on one device, for the comparison
        full = siso_segment(*_args(xd, 0, GL), state=std, chunk=128, policy_name="bf16")
        res += [full.y.float().cpu().numpy()] + [t.cpu().numpy() for t in full.state]
    q.put((rank, res))
    dist.barrier()
    dist.destroy_process_group()


GB, GH, GL, GN, GP, GNR = 2, 8, 1024, 128, 64, 32


def _gpu_case():
    from oracle import siso_oracle as O
    from tests.inputs import make_inputs

    x = make_inputs(GB, GH, GL, state_dim=GN, headdim=GP, n_angles=GNR, seed=7)
    g = torch.Generator().manual_seed(8)
    st = O.SISOState(ssm=torch.randn(GB, GH, GP, GN, generator=g, dtype=torch.float64) * 0.3,
                     k=torch.randn(GB, GH, GN, generator=g, dtype=torch.float64),
                     v=torch.randn(GB, GH, GP, generator=g, dtype=torch.float64),
                     phi=torch.rand(GB, GH, GNR, generator=g, dtype=torch.float64) * 6.0)
    return x, st


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_seq_parallel_on_two_gpus():
    from tests.metrics import rel_error

    world = 2
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_gpu_worker, args=(r, world, port, qu)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(qu.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    full_y, full_st = torch.from_numpy(res[0][5]), [torch.from_numpy(a) for a in res[0][6:]]
    per = GL // world
    for r in range(world):
        assert rel_error(torch.from_numpy(res[r][0]), full_y[:, :, r * per:(r + 1) * per]) < 2e-2, r
    last = [torch.from_numpy(a) for a in res[world - 1][1:5]]
    for name, a, b in zip(("ssm", "k", "v"), last[:3], full_st[:3]):
        assert rel_error(a, b) < 2e-2, name
    assert rel_error(last[3], full_st[3], angle=True) < 1e-4
