"""Multi-process batch sharding on CPU with the gloo backend (world size 2).

The per-rank compute here is the CPU oracle (the GPU library has no CPU path);
what is tested is the plumbing the benchmark uses on GPUs: contiguous shards
that cover the batch, MAX/SUM reductions of per-rank times, the optional
gather of (H, tau) shards, and failure of a rank surfacing as an error on the
others instead of a hang.
"""

from __future__ import annotations

import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

from gpumode_qr_b200 import sharding


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_ranges_cover_batch():
    for batch in (0, 1, 7, 8, 4096, 4097):
        for world in (1, 2, 3, 8):
            ranges = [sharding.shard_range(batch, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == batch
            for (s0, e0), (s1, _) in zip(ranges, ranges[1:]):
                assert e0 == s1
            sizes = [e - s for s, e in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.shard_range(4, 2, 2)


def _worker(rank, world, port, q, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import oracle
    from gpumode_qr_b200 import sharding as sh

    try:
        info = sh.init_from_env(backend="gloo", timeout_s=20.0)
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 failed on purpose (host-side)")
        A = torch.randn(7, 24, 24, generator=torch.Generator().manual_seed(0))

        def fn(x):
            H, tau = oracle.geqr2(x.numpy(), f64=True)
            return torch.from_numpy(H), torch.from_numpy(tau)

        s, e, H, tau = sh.run_sharded(fn, A, info)
        sh.barrier(info)
        tmax = sh.max_over_ranks(float(rank + 1), info)
        tsum = sh.sum_over_ranks(float(e - s), info)
        Hall = sh.gather_shards(H, A.shape[0], info)
        tall = sh.gather_shards(tau, A.shape[0], info)
        if rank == 0:
            Href, tref = fn(A)
            q.put(("ok", tmax, tsum, bool(torch.equal(Hall, Href)), bool(torch.equal(tall, tref))))
        sh.destroy(info)
    except Exception as ex:  # noqa: BLE001 - reported to the parent
        q.put(("err", rank, repr(ex)))


def _spawn(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    out = []
    while not q.empty():
        out.append(q.get())
    return out, alive


def test_two_rank_sharded_factorization_and_gather():
    out, alive = _spawn("ok")
    assert not alive
    oks = [o for o in out if o[0] == "ok"]
    assert oks, out
    _, tmax, tsum, h_eq, t_eq = oks[0]
    assert tmax == 2.0 and tsum == 7.0 and h_eq and t_eq


def test_failed_rank_surfaces_as_error_not_hang():
    out, alive = _spawn("fail")
    assert not alive, "a rank hung after its peer failed"
    errs = [o for o in out if o[0] == "err"]
    assert any(o[1] == 1 for o in errs)
    # rank 0 either errors in its first collective (peer gone) or times out
    assert any(o[1] == 0 for o in errs)
