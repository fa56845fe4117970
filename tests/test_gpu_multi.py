"""Long-context decode split across 2 GPUs, against one GPU and the oracle.

Both exchanges of the partials run on the same ranks: the NCCL all-gather + merge
and the NVLink exchange kernel (plain peer stores through CUDA IPC mappings, no
multicast); their outputs must be bit-identical.  Runs as two spawned ranks, one
per GPU; skipped when fewer than 2 GPUs are visible.  NVLS is disabled for the
test's NCCL communicator.  The one-rank tests of the exchange kernel run on one GPU.
"""

from __future__ import annotations

import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LENGTH = 3000


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    from oracle import kv_quant as kq

    rng = np.random.default_rng(22)
    k = kq.round_bf16(rng.standard_normal((1, 2, LENGTH, 256), dtype=np.float32))
    v = kq.round_bf16(rng.standard_normal((1, 2, LENGTH, 256), dtype=np.float32))
    q = kq.round_bf16(rng.standard_normal((2, 1, 8, 256), dtype=np.float32))       # two decode steps
    kn = kq.round_bf16(rng.standard_normal((1, 2, 1, 256), dtype=np.float32))      # token appended between them
    return k, v, q, kn


def _rank(rank, world, port, outdir):
    import torch.distributed as dist

    from optiz_qwen_b200.context_parallel import ContextParallelDecoder, PeerExchange

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    k, v, q, kn = _inputs()
    ex = PeerExchange(8, 256, rank=rank, world=world, device=dev, sites=1)
    dec = ContextParallelDecoder(2, 256, rank=rank, world=world, device=dev, exchange=ex)
    dec.prefill(torch.from_numpy(k).to(torch.bfloat16), torch.from_numpy(v).to(torch.bfloat16), capacity_tokens=16)

    ex2 = PeerExchange(8, 256, rank=rank, world=world, device=dev, sites=1)

    def both(qs):
        dec.exchange = None                                   # NCCL all-gather + oq_lse_merge
        a = dec.decode(qs).float().cpu().numpy()
        dec.exchange, dec.fused_exchange = ex, False          # standalone NVLink exchange kernel
        b = dec.decode(qs).float().cpu().numpy()
        c = dec.decode(qs).float().cpu().numpy()              # second call: the other slot parity
        dec.exchange, dec.fused_exchange = ex2, True          # exchange inside the split merge
        d = dec.decode(qs).float().cpu().numpy()
        e = dec.decode(qs).float().cpu().numpy()
        return np.stack([a, b, c, d, e])

    outs = [both(torch.from_numpy(q[0]).to(dev, torch.bfloat16))]
    knt = torch.from_numpy(kn).to(dev, torch.bfloat16)
    dec.append(knt, knt)
    outs.append(both(torch.from_numpy(q[1]).to(dev, torch.bfloat16)))
    status = int(ex.status.item()) | int(ex2.status.item())
    ex.close()
    ex2.close()
    np.save(os.path.join(outdir, f"out{rank}.npy"), np.stack(outs))
    np.save(os.path.join(outdir, f"status{rank}.npy"), np.array([status]))
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_long_context_split_over_two_gpus_matches_one_gpu_and_oracle():
    import torch.multiprocessing as mp

    from oracle import kv_quant as kq
    from oracle.attention import decode_attention
    from optiz_qwen_b200 import cabi
    from optiz_qwen_b200.compression.paged_kv import PagedKvState
    from tests._util import assert_attn_close

    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_rank, args=(2, _free_port(), d), nprocs=2, join=True)
        outs = [np.load(os.path.join(d, f"out{r}.npy")) for r in range(2)]
        statuses = [int(np.load(os.path.join(d, f"status{r}.npy"))[0]) for r in range(2)]
    assert statuses == [0, 0]
    k, v, q, kn = _inputs()
    # one GPU, whole cache
    pool = cabi.PagedKvPool(64, 2, 256, 64, "cuda")
    paged = PagedKvState(pool, 1, max_pages=60)
    paged.append(torch.from_numpy(k).cuda().to(torch.bfloat16), torch.from_numpy(v).cuda().to(torch.bfloat16))
    single0 = cabi.decode_attention_int4(torch.from_numpy(q[0]).cuda().to(torch.bfloat16), pool, paged.block_table,
                                         paged.seq_lens, 1 / 16).float().cpu().numpy()
    # oracle: fp32 attention over the dequantised cache (+ the appended token for step 2)
    kd = kq.dequantize_tokens_int4(*kq.quantize_tokens_int4(np.concatenate([k, kn], axis=2)))[0]
    vd = kq.dequantize_tokens_int4(*kq.quantize_tokens_int4(np.concatenate([v, kn], axis=2)))[0]
    ref0, _ = decode_attention(q[0], [kd[:, :LENGTH]], [vd[:, :LENGTH]], 1 / 16)
    ref1, _ = decode_attention(q[1], [kd], [vd], 1 / 16)
    for out in outs:           # out [step, exchange (nccl, standalone x2, in-merge x2), B, Hq, D]
        for x in range(5):
            assert_attn_close(out[0, x], ref0)
            assert_attn_close(out[1, x], ref1)
            assert_attn_close(out[0, x], single0)
        # the standalone exchange merges the same partials as the NCCL path: bit for bit
        for x in (1, 2):
            assert np.array_equal(out[:, 0], out[:, x]), f"standalone exchange call {x} differs from NCCL"
        # the in-merge exchange takes its partial from the split-merge kernel (another order of the
        # local split sums than the in-launch merge): repeatable, and within fp32 rounding of NCCL
        assert np.array_equal(out[:, 3], out[:, 4])
        np.testing.assert_allclose(out[:, 3], out[:, 0], rtol=2 ** -7, atol=1e-5)
    assert np.array_equal(outs[0], outs[1])        # every rank holds the same merged output


def test_one_rank_path_matches_partial_and_merge_and_oracle():
    """With one rank the decoder skips the fp32 partial, its packing and the merge: the attention
    kernel writes the output.  Both paths, before and after an append, against the oracle."""
    from oracle import kv_quant as kq
    from oracle.attention import decode_attention
    from optiz_qwen_b200.context_parallel import ContextParallelDecoder, PartialFns, context_parallel_attention
    from tests._util import assert_attn_close

    k, v, q, kn = _inputs()
    dec = ContextParallelDecoder(2, 256, rank=0, world=1, device="cuda")
    dec.prefill(torch.from_numpy(k).to(torch.bfloat16), torch.from_numpy(v).to(torch.bfloat16), capacity_tokens=16)
    kd = kq.dequantize_tokens_int4(*kq.quantize_tokens_int4(np.concatenate([k, kn], axis=2)))[0]
    vd = kq.dequantize_tokens_int4(*kq.quantize_tokens_int4(np.concatenate([v, kn], axis=2)))[0]
    refs = [decode_attention(q[0], [kd[:, :LENGTH]], [vd[:, :LENGTH]], 1 / 16)[0],
            decode_attention(q[1], [kd], [vd], 1 / 16)[0]]
    for step in range(2):
        if step == 1:
            knt = torch.from_numpy(kn).cuda().to(torch.bfloat16)
            dec.append(knt, knt)
        qt = torch.from_numpy(q[step]).cuda().to(torch.bfloat16)
        fast = dec.decode(qt)
        general = context_parallel_attention(qt, PartialFns(dec._partial, dec._merge))
        assert fast.dtype == torch.bfloat16 and fast.shape == qt.shape
        assert_attn_close(fast.float().cpu().numpy(), refs[step])
        assert_attn_close(general.float().cpu().numpy(), refs[step])
        assert_attn_close(fast.float().cpu().numpy(), general.float().cpu().numpy())


def test_exchange_kernel_one_rank_matches_lse_merge_in_graph_replays():
    """The exchange kernel with one rank: the merge of a single partial, bit-identical to
    oq_lse_merge, over eager calls and CUDA graph replays (the per-row call counters advance on
    the device)."""
    from optiz_qwen_b200 import cabi
    from optiz_qwen_b200.context_parallel import PeerExchange

    gen = torch.Generator(device="cuda").manual_seed(5)
    rows, d = 16, 256
    ex = PeerExchange(rows, d, rank=0, world=1, device="cuda", sites=2)
    part = torch.randn((rows, d), generator=gen, device="cuda")
    lse = torch.randn((rows,), generator=gen, device="cuda") * 4
    ref = cabi.lse_merge(part.view(1, rows, d), lse.view(1, rows), dtype=torch.bfloat16)
    for site in (0, 1, 0):
        out = ex.merge(site, part, lse)
        assert torch.equal(out, ref)
    out = torch.empty_like(ref)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        out.copy_(ex.merge(1, part, lse))
    for _ in range(3):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    assert int(ex.status.item()) == 0


@pytest.mark.parametrize("length", [3000, 40000])
def test_attention_with_exchange_one_rank_matches_oracle(length):
    """The attention launch whose split merge exchanges the rows (one rank): against the oracle
    and the plain launch, over eager calls and CUDA graph replays (both slot parities)."""
    from oracle import kv_quant as kq
    from oracle.attention import decode_attention
    from optiz_qwen_b200 import cabi
    from optiz_qwen_b200.compression.paged_kv import PagedKvState
    from optiz_qwen_b200.context_parallel import PeerExchange
    from tests._util import assert_attn_close

    rng = np.random.default_rng(length)
    k = kq.round_bf16(rng.standard_normal((1, 2, length, 256), dtype=np.float32))
    v = kq.round_bf16(rng.standard_normal((1, 2, length, 256), dtype=np.float32))
    q = kq.round_bf16(rng.standard_normal((1, 8, 256), dtype=np.float32))
    pages = -(-length // 64)
    pool = cabi.PagedKvPool(pages + 1, 2, 256, 64, "cuda")
    paged = PagedKvState(pool, 1, max_pages=pages)
    paged.append(torch.from_numpy(k).cuda().to(torch.bfloat16), torch.from_numpy(v).cuda().to(torch.bfloat16))
    kd = kq.dequantize_tokens_int4(*kq.quantize_tokens_int4(k))[0]
    vd = kq.dequantize_tokens_int4(*kq.quantize_tokens_int4(v))[0]
    ref, _ = decode_attention(q, [kd], [vd], 1 / 16)
    qt = torch.from_numpy(q).cuda().to(torch.bfloat16)
    ws = cabi.new_decode_workspace(1, 8, 2, pages, "cuda")
    ex = PeerExchange(8, 256, rank=0, world=1, device="cuda")
    plain = cabi.decode_attention_int4(qt, pool, paged.block_table, paged.seq_lens, 1 / 16, workspace=ws)

    def fused():
        return cabi.decode_attention_int4(qt, pool, paged.block_table, paged.seq_lens, 1 / 16, workspace=ws,
                                          exchange=ex.table(0), device_status=ex.status)

    outs = [fused(), fused()]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        g_out = fused()
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        outs.append(g_out.clone())
    assert int(ex.status.item()) == 0
    for o in outs:
        assert torch.equal(o, outs[0])
        assert_attn_close(o.float().cpu().numpy(), ref)
        assert_attn_close(o.float().cpu().numpy(), plain.float().cpu().numpy())
