"""Host side of the vocab-sharded path, on CPU with gloo ranks (no GPU).

The GPU path (vdxs_sample_sharded) splits each row's vocabulary into contiguous shards,
selects each shard's top-K with global indices, all-gathers the candidates and merges
them. These tests run the same decomposition with gloo ranks on the CPU:
- shard_range tiles [0, V) in rank order, also when V % world != 0;
- each rank applies the repetition penalty only to history ids it owns, in slot order
  (duplicates compound, Sampler.pas:285-303);
- each rank keeps its local top-K by (value desc, global index asc);
- the all-gathered union's top-K is the unsharded row's top-K from the oracle;
- broadcast_unique_id hands every rank the bytes made on rank 0.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _penalised_shard(x, hist, count, lo, hi, p):
    """Penalised copy of x[lo:hi]: per history slot, x>0 -> x/p, x<0 -> x*p, in fp32."""
    y = x[lo:hi].copy()
    pf = np.float32(p)
    for h in hist[:count]:
        if lo <= h < hi:
            v = y[h - lo]
            if v > 0:
                y[h - lo] = np.float32(v / pf)
            elif v < 0:
                y[h - lo] = np.float32(v * pf)
    return y


def _local_topk(y, lo, K):
    gidx = np.arange(len(y), dtype=np.int64) + lo
    order = np.lexsort((gidx, -y.astype(np.float64)))[:K]
    return y[order], gidx[order]


def _data(B, V, W, seed):
    rng = np.random.default_rng(seed)
    x = (rng.normal(size=(B, V)) * 4.0).astype(np.float32)
    x[:, rng.integers(0, V, size=8)] += 12.0
    hist = rng.integers(0, V, size=(B, W)).astype(np.int32)
    count = np.full(B, W, np.int32)
    return x, hist, count


def _worker(rank, world, port, B, V, K, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch
    import torch.distributed as dist
    from vindexllm_b200 import sampler
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        # The id the product would create with ncclGetUniqueId, made on rank 0 only.
        sampler.ShardComm.unique_id = staticmethod(lambda: bytes((i * 7 + 3) % 256 for i in range(128)))
        uid = sampler.broadcast_unique_id(rank)
        lo, hi = sampler.shard_range(V, world, rank)
        x, hist, count = _data(B, V, 512, seed=1234)
        vals = np.zeros((B, K), np.float32)
        idx = np.full((B, K), -1, np.int64)
        for b in range(B):
            y = _penalised_shard(x[b], hist[b], count[b], lo, hi, 1.1)
            v, i = _local_topk(y, lo, K)
            vals[b, :len(v)] = v
            idx[b, :len(i)] = i
        gv = [torch.zeros(B, K, dtype=torch.float32) for _ in range(world)]
        gi = [torch.zeros(B, K, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(gv, torch.from_numpy(vals))
        dist.all_gather(gi, torch.from_numpy(idx))
        merged = []
        for b in range(B):
            v = np.concatenate([t[b].numpy() for t in gv])
            i = np.concatenate([t[b].numpy() for t in gi])
            ok = i >= 0
            v, i = v[ok], i[ok]
            order = np.lexsort((i, -v.astype(np.float64)))[:K]
            merged.append(i[order])
        q.put((rank, uid, (lo, hi), np.stack(merged)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,V", [(2, 50001), (3, 40000)])
def test_sharded_decomposition_gloo(oracle_mod, world, V):
    import torch.multiprocessing as mp
    from vindexllm_b200.abi import default_config
    from vindexllm_b200 import abi
    B, K = 4, 40
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, V, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = {r: (uid, rng, m) for r, uid, rng, m in (q.get(timeout=240) for _ in range(world))}
    finally:
        for p in procs:
            p.join(timeout=60)
    for p in procs:
        assert p.exitcode == 0
    # shards tile the vocabulary in rank order
    ranges = [res[r][1] for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == V
    assert all(ranges[r][1] == ranges[r + 1][0] for r in range(world - 1))
    # every rank holds rank 0's id and the same merged candidates
    for r in range(world):
        assert res[r][0] == res[0][0]
        assert (res[r][2] == res[0][2]).all()
    # the merged top-K is the unsharded row's top-K (canonical oracle, no nucleus cut)
    x, hist, count = _data(B, V, 512, seed=1234)
    cfg = default_config(temperature=1.0, top_k=K, top_p=1.0, repeat_penalty=1.1, repeat_window=512)
    u = np.full(B, 0.5, np.float32)
    _, _, oi, _ = oracle_mod.sample_batch(cfg, x, u, hist, count, abi.TIES_CANONICAL, out_k=K)
    for b in range(B):
        assert set(oi[b].tolist()) == set(res[0][2][b].tolist())


def test_shard_range_edges():
    from vindexllm_b200.sampler import shard_range
    for V in (1, 7, 262144, 262145):
        for world in (1, 2, 3, 8):
            got = [shard_range(V, world, r) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == V
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            sizes = [h - l for l, h in got]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)
