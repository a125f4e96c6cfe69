"""Vocab-sharded sampling over 2+ GPUs (one process per GPU, NCCL all-gather of the
local top-k candidates). Equal, token for token, to the unsharded canonical result."""
import os

import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _worker(rank, world, uid, name, q):
    import torch
    from vindexllm_b200 import abi, synth
    from vindexllm_b200.sampler import SamplerContext, ShardComm, shard_range
    torch.cuda.set_device(rank)
    ctx = SamplerContext(rank, tie_mode=abi.TIES_CANONICAL)
    comm = ShardComm(ctx, world, rank, uid)
    cfg = synth.sampler_config(name)
    x = synth.make_logits(name, step=0, device=f"cuda:{rank}")
    V = x.shape[1]
    h, c = synth.make_history(name, step=0, device=f"cuda:{rank}")
    u = torch.as_tensor(synth.make_uniforms(name, 1, batch=x.shape[0])[0], device=f"cuda:{rank}")
    lo, hi = shard_range(V, world, rank)
    xs = x[:, lo:hi].contiguous()
    tok = comm.sample(cfg, xs, lo, V, u, h, c)
    torch.cuda.synchronize()
    ref = ctx.sample(cfg, x, u, h, c)
    torch.cuda.synchronize()
    q.put((rank, tok.cpu().numpy(), ref.cpu().numpy()))
    comm.close()
    ctx.close()


@pytest.mark.parametrize("name", ["c4", "c1"])
def test_sharded_equals_unsharded(name):
    import torch
    import torch.multiprocessing as mp
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    from vindexllm_b200.sampler import ShardComm
    uid = ShardComm.unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, uid, name, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    toks = {r: (t, ref) for r, t, ref in res}
    for r in range(world):
        assert (toks[r][0] == toks[0][0]).all()
        assert (toks[r][0] == toks[r][1]).all()
