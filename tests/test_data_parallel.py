"""Host logic of the batch-sharded multi-GPU path, on CPU with gloo ranks.

The solver is swapped for the CPU oracle here (there is no GPU), so these tests
cover the sharding, the flat gradient bucket and the SUM all-reduce: N ranks on
N shards must reproduce the single-process full-batch gradients.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import ltc_layer
import synth
from data_parallel import FlatGradBucket, shard_range, training_step
from oracle import ltc_oracle as orc


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg(B):
    return synth.LtcConfig("t", B, 3, 8, 6, 2, 0.5, 0.5)


def _model(cfg, p):
    m = ltc_layer.TrueLiquidTimeConstant(cfg.D, cfg.H, dt=cfg.dt, ode_unfolds=cfg.U)
    m.load_state_dict(p)
    return m


def _inputs(B):
    return (synth.make_params(8, 6, 0.5, 0.5, seed=5),
            torch.randn(B, 3, 8, generator=torch.Generator().manual_seed(9)))


def test_shard_range_covers_batch_exactly():
    for total in (1, 7, 16, 4096, 4097):
        for world in (1, 2, 3, 8):
            parts = [shard_range(total, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == total
            for (a, b), (c, d) in zip(parts, parts[1:]):
                assert b == c
            sizes = [b - a for a, b in parts]
            assert max(sizes) - min(sizes) <= 1


def test_flat_bucket_views_and_accumulation():
    ltc_layer.set_solver(orc.forward_loop)
    try:
        p, x = _inputs(3)
        m = _model(_cfg(3), p)
        bucket = FlatGradBucket(m.parameters())
        out, _ = m(x)
        out.sum().backward()
        bucket.check_views()
        first = bucket.flat.clone()
        out, _ = m(x)
        out.sum().backward()
        bucket.check_views()
        torch.testing.assert_close(bucket.flat, 2 * first)
        bucket.zero()
        assert bucket.flat.abs().sum() == 0
    finally:
        ltc_layer.set_solver(None)


def _worker(rank, world, port, B, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ltc_layer.set_solver(orc.forward_loop)
    p, x = _inputs(B)
    m = _model(_cfg(B), p)
    bucket = FlatGradBucket(m.parameters())
    opt = torch.optim.SGD(m.parameters(), lr=0.0)
    lo, hi = shard_range(B, rank, world)
    training_step(m, x[lo:hi], bucket, opt)
    out_q.put((rank, bucket.flat.detach().numpy().copy()))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,B", [(2, 6), (2, 5), (3, 7)])
def test_sharded_gradients_equal_full_batch(world, B):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = {r: torch.from_numpy(a) for r, a in (q.get(timeout=180) for _ in range(world))}
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    ltc_layer.set_solver(orc.forward_loop)
    try:
        p, x = _inputs(B)
        m = _model(_cfg(B), p)
        bucket = FlatGradBucket(m.parameters())
        out, _ = m(x)
        out.sum().backward()
    finally:
        ltc_layer.set_solver(None)
    for r in range(world):
        torch.testing.assert_close(res[r], bucket.flat, rtol=1e-5, atol=1e-5)
        assert torch.equal(res[r], res[0])
