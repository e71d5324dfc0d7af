"""Data-parallel gradient bucket on CPU ranks (gloo, world size 2): the
all-reduced sum of per-shard gradients equals the full-batch gradients, and a
rank that fails surfaces as an error instead of a hang."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mhc_ascend_b200.dp import GradBucket
from oracle import mhc_oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class OracleLayer(torch.nn.Module):
    """CPU stand-in with the layer's parameter set (the bucket is host logic)."""

    def __init__(self, params):
        super().__init__()
        for k in O.DYNAMIC_PARAM_ORDER:
            setattr(self, k, torch.nn.Parameter(params[k].clone()))

    def forward(self, x):
        return O.mhc_layer_dynamic(x, *[getattr(self, k) for k in O.DYNAMIC_PARAM_ORDER])


def _worker(rank, world, port, x, params, q, average):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layer = OracleLayer(params)
        shard = x.chunk(world)[rank]
        (layer(shard) ** 2).sum().backward()
        GradBucket(layer.parameters(), average=average).allreduce()
        # numpy copies pickle by value: a tensor would travel as a shared-memory
        # handle that can vanish when this process exits before the parent reads it
        q.put((rank, {k: p.grad.detach().numpy().copy() for k, p in layer.named_parameters()}))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("average", [False, True])
def test_bucket_allreduce_equals_full_batch(average):
    torch.manual_seed(0)
    B, n, C, world = 8, 4, 32, 2
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(B, n, C, generator=gen, dtype=torch.float64)
    params = {k: v.double() for k, v in O.make_dynamic_params(n, C, gen, alpha=0.5,
                                                              bias_std=0.5).items()}
    ref = OracleLayer(params)
    (ref(x) ** 2).sum().backward()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, x, params, q, average))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        for k, p in ref.named_parameters():
            expect = p.grad / world if average else p.grad
            torch.testing.assert_close(torch.from_numpy(results[r][k]), expect, rtol=1e-10,
                                       atol=1e-12)


def _shared_worker(rank, world, port, q):
    """Gradients already laid out as consecutive views of one buffer (what the
    fused backward produces) are all-reduced in place, without pack/unpack."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        params = [torch.nn.Parameter(torch.zeros(s)) for s in ((5,), (2, 3), (4,))]
        flat = torch.arange(15, dtype=torch.float32) + 100 * rank
        for p, g in zip(params, torch.split(flat, [5, 6, 4])):
            p.grad = g.view_as(p)
        bucket = GradBucket(params, average=True)
        shared = bucket._shared_flat()
        assert shared is not None and shared.data_ptr() == flat.data_ptr()
        bucket.allreduce()
        q.put((rank, flat.numpy().copy(), all(p.grad.data_ptr() >= flat.data_ptr() for p in params)))
    finally:
        dist.destroy_process_group()


def test_bucket_allreduces_shared_gradient_buffer_in_place():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shared_worker, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for pr in procs:
        pr.join(timeout=60)
    expect = torch.arange(15, dtype=torch.float32) + 50.0   # mean of rank 0 and rank 1 values
    for _, flat, views in res:
        assert torch.equal(torch.from_numpy(flat), expect)
        assert views


def _dying_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # a rank that leaves between steps
    lin = torch.nn.Linear(4, 4)
    lin(torch.randn(2, 4)).sum().backward()
    try:
        GradBucket(lin.parameters()).allreduce()
        q.put("no error")
    except Exception as e:  # gloo reports the lost peer / timeout
        q.put("error: " + type(e).__name__)


def test_lost_rank_surfaces_as_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    msg = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert msg.startswith("error"), msg
