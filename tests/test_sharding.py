"""Multi-rank host logic: (batch, KV head) unit partition, repacking, 2-rank gloo run."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import swa_oracle as orc
from tests._pkg import submodule


def test_plan_units_covers_every_unit_once():
    sh = submodule("sharding")
    for b, hkv, world in [(4, 8, 1), (4, 8, 3), (1, 8, 8), (2, 3, 4), (1, 1, 2)]:
        plans = sh.plan_units(b, hkv, world)
        flat = [u for p in plans for u in p]
        assert sorted(flat) == sh.all_units(b, hkv)
        sizes = [len(p) for p in plans]
        assert max(sizes) - min(sizes) <= 1


def test_unit_batch_round_trip_and_independence():
    sh = submodule("sharding")
    g = torch.Generator().manual_seed(0)
    q = torch.randn(2, 6, 40, 16, generator=g)
    k = torch.randn(2, 3, 40, 16, generator=g)
    v = torch.randn(2, 3, 40, 16, generator=g)
    do = torch.randn(2, 6, 40, 16, generator=g)
    units = [(1, 2), (0, 0), (1, 0)]
    qu, ku, vu, dou = sh.to_unit_batch(q, k, v, units, do)
    assert qu.shape == (3, 2, 40, 16) and ku.shape == (3, 1, 40, 16)
    # a unit computed alone equals its slice of the full problem
    full = orc.backward(q, k, v, do, 7, 2)
    part = orc.backward(qu, ku, vu, dou, 7, 2)
    for f, p in zip(full, part):
        back = sh.from_unit_batch(p.to(f.dtype), units, 2, 3)
        h = f.shape[1] // 3
        for j, (b_, kh) in enumerate(units):
            assert torch.allclose(back[b_, kh * h:(kh + 1) * h], f[b_, kh * h:(kh + 1) * h])


def _oracle_compute(q, k, v, do, w, s):
    return tuple(t.to(q.dtype) for t in orc.backward(q, k, v, do, w, s))


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = submodule("sharding")
        g = torch.Generator().manual_seed(3)
        q = torch.randn(3, 4, 50, 16, generator=g)
        k = torch.randn(3, 2, 50, 16, generator=g)
        v = torch.randn(3, 2, 50, 16, generator=g)
        do = torch.randn(3, 4, 50, 16, generator=g)
        res = sh.sharded_backward(q, k, v, do, 9, 3, _oracle_compute)
        ref = orc.backward(q, k, v, do, 9, 3)
        ok = all(torch.allclose(a, b.to(a.dtype), atol=1e-5) for a, b in zip(res, ref))
        out[rank] = 1 if ok else 0
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_sharded_backward_matches_single_process():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    out = ctx.Array("i", [0, 0])
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert list(out) == [1, 1]


# ---------------------------------------------------------------------------------------
# sequence split with a K/V halo (seqsplit.py): the exchange protocol on gloo CPU ranks, the
# local compute being the fp64 oracle
# ---------------------------------------------------------------------------------------

def _orc_fwd(q, k, v, w, s, scale):
    return orc.forward(q, k, v, w, s, scale)


def _orc_bwd(q, k, v, o, lse, do, w, s, scale):
    return orc.backward(q, k, v, do, w, s, scale)[1:]


def _seq_worker(rank, world, port, out, L, w, s):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ss = submodule("seqsplit")
        g = torch.Generator().manual_seed(11)
        q = torch.randn(2, 4, L, 16, generator=g, dtype=torch.float64)
        k = torch.randn(2, 2, L, 16, generator=g, dtype=torch.float64)
        v = torch.randn(2, 2, L, 16, generator=g, dtype=torch.float64)
        do = torch.randn(2, 4, L, 16, generator=g, dtype=torch.float64)
        a, b = ss.split_bounds(L, world)[rank]
        o, st = ss.seq_sharded_forward(q[:, :, a:b], k[:, :, a:b], v[:, :, a:b], L, w, s,
                                       fwd_fn=_orc_fwd)
        dq, dk, dv = ss.seq_sharded_backward(st, do[:, :, a:b], bwd_fn=_orc_bwd)
        ref = orc.backward(q, k, v, do, w, s)
        ok = all(torch.allclose(x, r[:, :, a:b], atol=1e-9)
                 for x, r in zip((o, dq, dk, dv), ref))
        out[rank] = 1 if ok else 0
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,L,w,s", [(2, 700, 50, 3), (3, 900, 129, 4), (2, 300, 1, 0),
                                         (3, 1000, 128, 16)])
def test_seq_split_gloo_matches_single_process(world, L, w, s):
    import socket
    sock = socket.socket()
    sock.bind(("127.0.0.1", 0))
    port = sock.getsockname()[1]
    sock.close()
    ctx = mp.get_context("spawn")
    out = ctx.Array("i", [0] * world)
    procs = [ctx.Process(target=_seq_worker, args=(r, world, port, out, L, w, s))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    assert list(out) == [1] * world


def test_seq_split_layout_rules():
    ss = submodule("seqsplit")
    assert ss.split_bounds(1000, 3) == [(0, 384), (384, 768), (768, 1000)]
    start, end, halo, pre = ss.layout(131072, 8, 3, 128, 4)
    assert (start, end, halo, pre) == (3 * 16384, 4 * 16384, 127, 256)
    with pytest.raises(ValueError):
        ss.layout(1024, 4, 2, 512, 0)      # halo longer than the previous rank's rows
    with pytest.raises(ValueError):
        ss.layout(1024, 2, 1, 512, 4)      # halo would reach the sink rows
