"""Multi-rank host logic on CPU (gloo, world size 2): each rank computes the
attention of its head shard with the oracle, the shards are all-gathered and
must reproduce the single-rank result bit for bit; the bench's max-over-ranks
timing reduction is exercised on the same process group."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from gfx906_fa_shard import head_shard


def test_head_shard_ranges():
    s = [head_shard(48, 8, 4, r) for r in range(4)]
    assert [(x.q0, x.q1, x.kv0, x.kv1) for x in s] == [(0, 12, 0, 2), (12, 24, 2, 4), (24, 36, 4, 6), (36, 48, 6, 8)]
    # more ranks than kv heads: each kv head replicated, query heads split
    r = [head_shard(48, 4, 8, k) for k in range(8)]
    assert [(x.q0, x.kv0) for x in r] == [(0, 0), (6, 0), (12, 1), (18, 1), (24, 2), (30, 2), (36, 3), (42, 3)]
    for x in r:                                   # every query head reads its own kv head
        assert all(q * 4 // 48 == x.kv0 for q in range(x.q0, x.q1))
    with pytest.raises(ValueError):
        head_shard(48, 8, 5, 0)


def _problem():
    rng = np.random.default_rng(11)
    Hq, Hkv, D, bs = 8, 2, 128, 16
    lens = np.array([70, 33], np.int32)
    nb = [(int(L) + bs - 1) // bs for L in lens]
    NB = sum(nb)
    bt = np.full((2, max(nb)), -1, np.int32)
    bt[0, :nb[0]] = np.arange(nb[0])
    bt[1, :nb[1]] = nb[0] + np.arange(nb[1])
    T = int(lens.sum())
    key = rng.standard_normal((T, Hkv, D)).astype(np.float16)
    val = rng.standard_normal((T, Hkv, D)).astype(np.float16)
    slots = np.concatenate([bt[b, np.arange(L) // bs] * bs + np.arange(L) % bs for b, L in enumerate(lens)])
    k_cache = np.zeros((NB, bs, Hkv, O.row_bytes(D)), np.uint8)
    O.reshape_and_cache(key, slots.astype(np.int64), k_cache)
    v_cache = np.zeros((NB, bs, Hkv, D), np.float16)
    O.store_v16(val, slots.astype(np.int64), v_cache)
    q = rng.standard_normal((2, Hq, D)).astype(np.float32)          # one decode token per sequence
    return q, k_cache, v_cache, bt, lens, Hq, Hkv


def _attend(q, k_cache, v_cache, bt, lens, Hkv):
    return O.attention_paged(q, None, np.arange(2, dtype=np.int32), np.ones(2, np.int32),
                             np.ascontiguousarray(k_cache), np.ascontiguousarray(v_cache), bt, lens,
                             0.088, Hkv)


def _worker(rank, world, port, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    q, k_cache, v_cache, bt, lens, Hq, Hkv = _problem()
    s = head_shard(Hq, Hkv, world, rank)
    # the rank's own cache holds only its kv heads, as under vLLM TP
    out = _attend(q[:, s.q0:s.q1], k_cache[:, :, s.kv0:s.kv1], v_cache[:, :, s.kv0:s.kv1], bt, lens,
                  s.num_heads_kv)
    parts = [torch.zeros_like(torch.from_numpy(out)) for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(out))
    t = torch.tensor([float(rank + 1)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)            # bench.py's max-over-ranks timing
    if rank == 0:
        ret.put((torch.cat(parts, dim=1).numpy(), float(t.item())))
    dist.barrier()
    dist.destroy_process_group()


def test_head_sharded_attention_gloo():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ret)) for r in range(2)]
    for p in procs:
        p.start()
    got, tmax = ret.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q, k_cache, v_cache, bt, lens, Hq, Hkv = _problem()
    full = _attend(q, k_cache, v_cache, bt, lens, Hkv)
    assert np.array_equal(got, full)
    assert tmax == 2.0
