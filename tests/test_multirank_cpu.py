"""Multi-rank host logic of bench.py on CPU with the gloo backend (world size 2): each rank
gets identical model weights but its own synthetic batch (weak scaling, no data-path
collective), and the timing reduction takes the maximum over ranks."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        import bdh_model

        # the reduction used for the reported time
        t = bench.max_over_ranks(float(10 + rank), world, torch.device("cpu"))
        # weights identical across ranks, inputs different
        cfg = bdh_model.BDHConfig(n_layer=1, n_embd=16, n_head=2, mlp_internal_dim_multiplier=2,
                                  vocab_size=32, dropout=0.0)
        torch.manual_seed(1002)
        m = bdh_model.BDH(cfg)
        wsum = torch.tensor([float(m.encoder.sum())])
        g = torch.Generator().manual_seed(bench.rank_seed(2002, rank))
        idx = torch.randint(0, 32, (2, 8), generator=g)
        ws = [torch.zeros(1) for _ in range(world)]
        dist.all_gather(ws, wsum)
        xs = [torch.zeros(2, 8, dtype=torch.long) for _ in range(world)]
        dist.all_gather(xs, idx)
        # the untimed cross-rank verification: same batch on every rank, checksums gathered
        m.attn._attn_impl_override = "eager"
        gv = torch.Generator().manual_seed(4242)
        iv = torch.randint(0, 32, (2, 8), generator=gv)
        with torch.no_grad():
            chk = bench.cross_rank_check(lambda: m(iv)[0], world, torch.device("cpu"))
        q.put((rank, t, [float(w) for w in ws], bool(torch.equal(xs[0], xs[1])), chk["identical"]))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_weak_scaling_logic():
    import sys

    from conftest import REPO

    sys.path.insert(0, str(REPO))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=5) for _ in range(2))
    for rank, t, ws, same_inputs, identical in res:
        assert t == 11.0          # max over ranks
        assert ws[0] == ws[1]     # replicated weights
        assert not same_inputs    # per-rank batches differ
        assert identical          # the verification batch gives the same logits on every rank
