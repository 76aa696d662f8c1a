"""The N > 1 host logic on CPU: world_size-2 gloo ranks shard the weights over
N and the attention / KDA inputs over kv-head groups, compute each shard with
the CPU oracle (standing in for the per-GPU kernel), and the all-gather (or the
head concatenation) must reproduce the single-rank result exactly."""
import os
import socket

import numpy as np
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


def _worker(rank, world, port, results):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(here))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "triton-metal_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from b200kern import sharding
    from b200kern.quant import pack_int4_gptq, unpack_int4_gptq
    from oracle import attention as oatt, kda as okda, quant as oq
    g = torch.Generator().manual_seed(0)
    # --- W4A16, N sharded, all-gathered ---
    M, K, N, G = 3, 256, 200, 128
    x = torch.randn(M, K, generator=g)
    q = torch.randint(0, 16, (K, N), generator=g)
    s = torch.rand(K // G, N, generator=g) * 0.02 + 1e-3
    qw, ss, _, (a, b) = sharding.shard_int4(pack_int4_gptq(q), s, world=world, rank=rank)
    part = oq.int4_matmul(x.numpy(), unpack_int4_gptq(qw).numpy(), ss.numpy(), None, G)
    full = sharding.all_gather_columns(torch.from_numpy(part))
    ok_w4 = np.array_equal(full.numpy(), oq.int4_matmul(x.numpy(), q.numpy(), s.numpy(), None, G))
    # --- W8A16, N sharded ---
    w8 = torch.randint(-127, 128, (N, K), generator=g).to(torch.int8)
    s8 = torch.rand(N, generator=g)
    w_, s_, _, _ = sharding.shard_int8(w8, s8, world=world, rank=rank)
    full8 = sharding.all_gather_columns(torch.from_numpy(oq.int8_matmul(x.numpy(), w_.numpy(), s_.numpy())))
    ok_w8 = np.array_equal(full8.numpy(), oq.int8_matmul(x.numpy(), w8.numpy(), s8.numpy()))
    # --- GQA attention, kv-head-group sharded ---
    qa = torch.randn(2, 8, 16, 32, generator=g)
    ka = torch.randn(2, 4, 16, 32, generator=g)
    va = torch.randn(2, 4, 16, 32, generator=g)
    qs, ks, vs, (ha, hb) = sharding.shard_heads(qa, ka, va, world, rank)
    oa = oatt.attention(qs.numpy(), ks.numpy(), vs.numpy(), causal=True)
    ref = oatt.attention(qa.numpy(), ka.numpy(), va.numpy(), causal=True)[:, ha * 2: hb * 2]
    ok_fa = np.array_equal(oa, ref)
    # --- KDA, head sharded ([B, T, H, D]) ---
    kq, kk, kv, kg, kb = okda.make_inputs(1, 32, 4, 16, seed=3)
    t = torch.from_numpy
    qh, kh, vh, (h0, h1) = sharding.shard_heads(t(kq), t(kk), t(kv), world, rank, head_dim=2)
    ok_, _ = okda.recurrent(qh.numpy(), kh.numpy(), vh.numpy(), kg[:, :, h0:h1], kb[:, :, h0:h1])
    ref_k, _ = okda.recurrent(kq, kk, kv, kg, kb)
    ok_kda = np.allclose(ok_, ref_k[:, :, h0:h1], rtol=0, atol=1e-12)
    # --- equal-width shards: one all_gather_into_tensor, then the [M, N] view ---
    Ne = 256
    qe = torch.randint(0, 16, (K, Ne), generator=g)
    se = torch.rand(K // G, Ne, generator=g) * 0.02 + 1e-3
    qwe, sse, _, _ = sharding.shard_int4(pack_int4_gptq(qe), se, world=world, rank=rank)
    parte = torch.from_numpy(oq.int4_matmul(x.numpy(), unpack_int4_gptq(qwe).numpy(), sse.numpy(), None, G))
    stacked = sharding.all_gather_columns_stacked(parte)
    ok_st = stacked.shape == (world, M, Ne // world) and np.array_equal(
        sharding.columns_from_stacked(stacked).numpy(), oq.int4_matmul(x.numpy(), qe.numpy(), se.numpy(), None, G))
    ok_w4 = ok_w4 and ok_st
    results[rank] = (ok_w4, ok_w8, ok_fa, ok_kda, (a, b))
    dist.barrier()
    dist.destroy_process_group()


def test_shard_range_covers_everything():
    from b200kern.sharding import shard_range
    for n, world, align in [(11008, 8, 8), (14336, 8, 256), (32, 3, 1), (16, 8, 8)]:
        spans = [shard_range(n, world, r, align) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
        assert all((b - a) % align == 0 for a, b in spans)


def test_two_gloo_ranks_match_single_rank():
    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(_worker, args=(2, _free_port(), results), nprocs=2, join=True)
    assert set(results.keys()) == {0, 1}
    for rank in (0, 1):
        ok_w4, ok_w8, ok_fa, ok_kda, _ = results[rank]
        assert ok_w4 and ok_w8 and ok_fa and ok_kda, results[rank]
    assert results[0][4][1] == results[1][4][0]
