"""Host logic of the multi-GPU paths on CPU ranks (gloo, world size 2).

* long context: each rank attends over its page-aligned KV range, the partials
  travel through one all-gather and are merged by log-sum-exp; the result equals
  attention over the whole cache (the compute here is the oracle; on GPUs it is
  the sm_100a kernels behind the same PartialFns seam);
* batched serving: every rank computes the same byte-balanced sharding;
* failure: a rank that dies before the collective makes its peer's collective
  fail with an error instead of hanging.
"""

from __future__ import annotations

import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _long_context_rank(rank, world, port, outdir):
    from oracle import attention as oattn
    from oracle import kv_quant as kq
    from optiz_qwen_b200.context_parallel import PartialFns, context_parallel_attention, kv_ranges

    _init(rank, world, port)
    rng = np.random.default_rng(2)
    length = 1000
    cache = kq.fill_paged_cache(rng, [length], 2, 256, 64, seed_pages=2)
    k, v = cache.gather(0)
    q = kq.round_bf16(rng.standard_normal((1, 8, 256), dtype=np.float32))
    lo, hi = kv_ranges(length, world)[rank]

    def partial(qt):
        o, l = oattn.decode_attention(qt.numpy(), [k[:, lo:hi]], [v[:, lo:hi]], 256 ** -0.5)
        return torch.from_numpy(o), torch.from_numpy(l)

    def merge(po, pl):
        o, _ = oattn.lse_merge(po.numpy(), pl.numpy())
        return torch.from_numpy(o)

    out = context_parallel_attention(torch.from_numpy(q), PartialFns(partial, merge))
    np.save(os.path.join(outdir, f"cp{rank}.npy"), out.numpy())
    dist.destroy_process_group()


def test_long_context_merge_over_two_ranks():
    from oracle import attention as oattn
    from oracle import kv_quant as kq

    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_long_context_rank, args=(2, _free_port(), d), nprocs=2, join=True)
        outs = [np.load(os.path.join(d, f"cp{r}.npy")) for r in range(2)]
    rng = np.random.default_rng(2)
    cache = kq.fill_paged_cache(rng, [1000], 2, 256, 64, seed_pages=2)
    k, v = cache.gather(0)
    q = kq.round_bf16(rng.standard_normal((1, 8, 256), dtype=np.float32))
    ref, _ = oattn.decode_attention(q, [k], [v], 256 ** -0.5)
    for out in outs:
        np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-6)


def test_kv_ranges_cover_and_align():
    from optiz_qwen_b200.context_parallel import kv_ranges

    for length in (0, 1, 63, 64, 65, 1000, 131072):
        for world in (1, 2, 4, 8):
            rs = kv_ranges(length, world)
            assert rs[0][0] == 0 and rs[-1][1] == length
            for (a, b), (c, _) in zip(rs, rs[1:]):
                assert b == c and a <= b
            assert all(lo % 64 == 0 for lo, hi in rs if hi > lo)


def _sharding_rank(rank, world, port, outdir):
    from optiz_qwen_b200.serving import shard_by_cost

    _init(rank, world, port)
    lengths = np.random.default_rng(3).integers(256, 8193, size=1024).tolist()
    shards = shard_by_cost(lengths, world)
    mine = torch.tensor(shards[rank], dtype=torch.int64)
    sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(sizes, torch.tensor([len(mine)]))
    gathered = [torch.zeros(int(s.item()), dtype=torch.int64) for s in sizes]
    dist.all_gather(gathered, mine)
    np.save(os.path.join(outdir, f"sh{rank}.npy"), torch.cat(gathered).numpy())
    dist.destroy_process_group()


def test_sequence_sharding_is_consistent_and_complete():
    from optiz_qwen_b200.serving import shard_by_cost, shard_loads

    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_sharding_rank, args=(2, _free_port(), d), nprocs=2, join=True)
        got = [np.load(os.path.join(d, f"sh{r}.npy")) for r in range(2)]
    assert np.array_equal(got[0], got[1])
    assert sorted(got[0].tolist()) == list(range(1024))
    lengths = np.random.default_rng(3).integers(256, 8193, size=1024).tolist()
    for world in (2, 4, 8):
        loads = shard_loads(lengths, shard_by_cost(lengths, world))
        assert max(loads) / min(loads) < 1.01


def _dying_rank(rank, world, port, outdir):
    _init(rank, world, port, timeout_s=10)
    if rank == 1:
        os._exit(0)                      # leaves without joining the collective
    try:
        t = torch.zeros(4)
        out = torch.zeros(8)
        dist.all_gather_into_tensor(out, t)
        status = "no error"
    except Exception as exc:             # the surviving rank must see an error, not hang
        status = f"error: {type(exc).__name__}"
    with open(os.path.join(outdir, "status.txt"), "w") as f:
        f.write(status)


def test_rank_failure_surfaces_as_an_error():
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_dying_rank, args=(r, 2, port, d)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        alive = [p for p in procs if p.is_alive()]
        for p in alive:
            p.kill()
        assert not alive, "a rank hung"
        with open(os.path.join(d, "status.txt")) as f:
            assert f.read().startswith("error")
