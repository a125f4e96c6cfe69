"""Vocab-sharded sampling over 2, 4 and 8 GPUs (one process per GPU, NCCL all-gather of
the local top-k candidates): every rank's tokens equal the CPU oracle's canonical
result (lowest-index ties, the order that composes across contiguous shards) on the
full, unsharded rows. c4 is the benchmark's sharded configuration; c1 routes each
row's 512-id history to the shard that owns each id. Skips when fewer GPUs are visible."""
import numpy as np
import pytest

from vindexllm_b200 import abi

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _worker(rank, world, uid, name, q):
    try:
        import torch
        from vindexllm_b200 import synth
        from vindexllm_b200.sampler import SamplerContext, ShardComm, shard_range
        torch.cuda.set_device(rank)
        dev = f"cuda:{rank}"
        ctx = SamplerContext(rank, tie_mode=abi.TIES_CANONICAL)
        comm = ShardComm(ctx, world, rank, uid)
        cfg = synth.sampler_config(name)
        x = synth.make_logits(name, step=0, device=dev)
        V = x.shape[1]
        h, c = synth.make_history(name, step=0, device=dev)
        lo, hi = shard_range(V, world, rank)
        xs = x[:, lo:hi].contiguous()
        del x
        toks = []
        for step in range(2):  # two calls in a row reuse the communicator and workspace
            u = torch.as_tensor(synth.make_uniforms(name, step + 1, batch=xs.shape[0])[step], device=dev)
            toks.append(comm.sample(cfg, xs, lo, V, u, h, c).cpu().numpy())
        ctx.device_status()
        q.put((rank, "ok", toks))
        comm.close()
        ctx.close()
    except BaseException as exc:  # report instead of leaving the parent waiting
        q.put((rank, "error", repr(exc)))


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("name", ["c4", "c1"])
def test_sharded_equals_oracle(name, world, oracle_mod):
    import torch
    import torch.multiprocessing as mp
    from vindexllm_b200 import synth
    from tests.gpu_helpers import NTHREADS, to_host_bits
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from vindexllm_b200.sampler import ShardComm
    uid = ShardComm.unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, uid, name, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    errs = [(r, m) for r, s, m in res if s != "ok"]
    assert not errs, errs
    toks = {r: t for r, _, t in res}
    # The oracle on the full rows (generated on the host from the same seeds).
    cfg = synth.sampler_config(name)
    x = to_host_bits(synth.make_logits(name, step=0, device="cuda:0"))
    h, c = synth.make_history(name, step=0, device="cuda:0")  # the workers' generator stream
    h, c = (None, None) if h is None else (h.cpu(), c.cpu())
    for step in range(2):
        u = synth.make_uniforms(name, step + 1, batch=x.shape[0])[step]
        want, _, _, _ = oracle_mod.sample_batch(cfg, x, u, None if h is None else h.numpy(),
                                                None if c is None else c.numpy(), abi.TIES_CANONICAL,
                                                nthreads=NTHREADS, diag=False)
        for r in range(world):
            bad = np.nonzero(toks[r][step] != want)[0]
            assert len(bad) == 0, f"{name} world {world} rank {r} step {step}: {len(bad)} mismatches, rows {bad[:5]}"
