"""Data-parallel gradient averaging (the counterpart of ``jax.lax.pmean`` in
``train.py:427-451``) with two gloo ranks on the CPU: bucketed all-reduce hooks fire
during backward and leave every rank with the mean gradient."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "mamba3-siso-tpu_b200"))
    from mamba3_b200.train import GradBucketer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)
    ws = [torch.randn(5, 7, requires_grad=True), torch.randn(7, requires_grad=True), torch.randn(7, 3, requires_grad=True)]
    bk = GradBucketer(ws, bucket_bytes=64)
    x = torch.randn(4, 5, generator=torch.Generator().manual_seed(rank + 1))
    loss = ((x @ ws[0] + ws[1]) @ ws[2]).pow(2).sum()
    loss.backward()
    bk.finish()
    # numpy copies travel by value (a shared tensor's storage can vanish with the process)
    q.put((rank, [w.grad.clone().numpy() for w in ws]))
    dist.barrier()
    dist.destroy_process_group()


def test_bucketed_allreduce_mean_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r: [torch.from_numpy(a) for a in gs] for r, gs in (q.get(timeout=120) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # expected: mean over the two ranks' local grads
    torch.manual_seed(0)
    ws = [torch.randn(5, 7, requires_grad=True), torch.randn(7, requires_grad=True), torch.randn(7, 3, requires_grad=True)]
    grads = []
    for r in range(2):
        x = torch.randn(4, 5, generator=torch.Generator().manual_seed(r + 1))
        g = torch.autograd.grad(((x @ ws[0] + ws[1]) @ ws[2]).pow(2).sum(), ws)
        grads.append(g)
    for i in range(3):
        want = (grads[0][i] + grads[1][i]) / 2
        assert torch.allclose(res[0][i], want, atol=1e-5)
        assert torch.allclose(res[1][i], want, atol=1e-5)
