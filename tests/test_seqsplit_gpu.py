"""GPU check of the sequence split with a K/V halo (seqsplit.py): two ranks, each running this
library's kernels on its local problem, against the single-process result of the dense entry
point on the whole sequence.

With two or more GPUs the ranks use one GPU each and NCCL; with one GPU both ranks share it and
exchange through a gloo group (host-staged copies).  Neither rank's kernels wait on the other's.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests._pkg import pkg, submodule

pytestmark = pytest.mark.gpu
TOL = {torch.float16: 2e-3, torch.bfloat16: 1.5e-2}


def _rel(x, r):
    x, r = x.double().cpu(), r.double().cpu()
    return ((x - r).abs().max() / r.abs().max().clamp_min(1e-30)).item()


def _worker(rank, world, port, out, L, w, s, dtype_name):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    multi = torch.cuda.device_count() >= world
    dev = torch.device("cuda", rank if multi else 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl" if multi else "gloo", rank=rank, world_size=world,
                            device_id=dev if multi else None)
    try:
        dtype = getattr(torch, dtype_name)
        ss = submodule("seqsplit")
        g = torch.Generator().manual_seed(21)
        q, do = (torch.randn(1, 8, L, 64, generator=g).to(dtype) for _ in range(2))
        k, v = (torch.randn(1, 2, L, 64, generator=g).to(dtype) for _ in range(2))
        # whole sequence, one process
        qf, kf, vf = (t.to(dev).requires_grad_() for t in (q, k, v))
        of = pkg().flash_swda_with_sink(qf, kf, vf, w, s)
        of.backward(do.to(dev))
        a, b = ss.split_bounds(L, world)[rank]
        qs, ks, vs = (t[:, :, a:b].contiguous().to(dev).requires_grad_() for t in (q, k, v))
        o = ss.SeqShardedSWDA.apply(qs, ks, vs, L, w, s)
        o.backward(do[:, :, a:b].to(dev))
        errs = [_rel(x, r[:, :, a:b]) for x, r in
                zip((o, qs.grad, ks.grad, vs.grad), (of, qf.grad, kf.grad, vf.grad))]
        out[rank] = 1 if max(errs) <= TOL[dtype] else 0
        if not out[rank]:
            print("rank", rank, "errors", errs, flush=True)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("L,w,s,dtype", [(2048, 128, 4, "float16"), (3000, 300, 16, "bfloat16"),
                                         (1536, 1, 0, "float16")])
def test_seq_split_two_ranks_match_whole_sequence(L, w, s, dtype):
    sock = socket.socket()
    sock.bind(("127.0.0.1", 0))
    port = sock.getsockname()[1]
    sock.close()
    ctx = mp.get_context("spawn")
    out = ctx.Array("i", [0, 0])
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out, L, w, s, dtype)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    assert list(out) == [1, 1]
