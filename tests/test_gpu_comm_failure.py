"""Failure detection on the vocab-sharded path's communicator (the one collective this
library adds; the reference has none). Both failures are made on the host and no GPU is
left waiting: a rank that never joins the communicator (the others' creation must end in
VDXS_E_TIMEOUT within the limit), and a rank that leaves between two sharded steps with
none of its work in flight (it drops its own communicator and tells the others on the
host; the survivor learns it before its next launch, aborts its communicator, and the
next call must refuse without launching anything).
Ranks run as spawned processes with NVLS off."""
import os
import time

import pytest

from vindexllm_b200 import abi

pytestmark = pytest.mark.gpu


def _child_env():
    os.environ["NCCL_NVLS_ENABLE"] = "0"


def _never_joins_worker(q, timeout_ms):
    try:
        _child_env()
        import torch
        from vindexllm_b200.sampler import SamplerContext, ShardComm, VdxsError
        torch.cuda.set_device(0)
        ctx = SamplerContext(0)
        uid = ShardComm.unique_id()
        t0 = time.monotonic()
        try:
            ShardComm(ctx, 2, 0, uid, timeout_ms=timeout_ms)  # rank 1 never calls
            q.put(("no-error", time.monotonic() - t0, None))
            return
        except VdxsError as exc:
            took = time.monotonic() - t0
            code = exc.code
        # The context is still usable afterwards: a one-rank communicator works.
        c1 = ShardComm(ctx, 1, 0, ShardComm.unique_id(), timeout_ms=timeout_ms)
        c1.close()
        ctx.close()
        q.put(("ok", took, code))
    except BaseException as exc:
        q.put(("error", 0.0, repr(exc)))


def test_comm_create_times_out_when_a_rank_never_joins():
    import torch
    import torch.multiprocessing as mp
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    p = mpc.Process(target=_never_joins_worker, args=(q, 3000))
    p.start()
    status, took, code = q.get(timeout=300)
    p.join(timeout=60)
    assert status == "ok", (status, code)
    assert code == abi.E_TIMEOUT
    assert took < 3.0 + 5.0, f"creation gave up after {took:.1f} s (limit 3 s)"


def _leaver_worker(rank, world, uid, q, left):
    try:
        _child_env()
        import torch
        from vindexllm_b200 import synth
        from vindexllm_b200.sampler import SamplerContext, ShardComm, VdxsError, shard_range
        torch.cuda.set_device(rank)
        dev = f"cuda:{rank}"
        ctx = SamplerContext(rank, tie_mode=abi.TIES_CANONICAL)
        comm = ShardComm(ctx, world, rank, uid, timeout_ms=20000)
        q.put((rank, "progress", "communicator created"))
        cfg = synth.sampler_config("c4")
        x = synth.make_logits("c4", step=0, batch=16, device=dev)
        V = x.shape[1]
        lo, hi = shard_range(V, world, rank)
        xs = x[:, lo:hi].contiguous()
        u = torch.as_tensor(synth.make_uniforms("c4", 1, batch=16)[0], device=dev)
        tok = comm.sample(cfg, xs, lo, V, u)
        comm.wait(timeout_ms=20000)  # step 1 completed on this rank, nothing left in flight
        first = tok.cpu().numpy()
        q.put((rank, "progress", "step 1 done"))
        if rank == 1:
            # This rank leaves between steps: nothing of it is in flight; it drops its own
            # communicator (a local abort) and tells the others on the host.
            torch.cuda.synchronize()
            comm.abort()
            comm.close()
            ctx.close()
            q.put((rank, "left", first.tolist()))
            left.set()
            return
        # Rank 0 learns on the host that its peer left, before its next launch.
        if not left.wait(timeout=120):
            q.put((rank, "error", "peer never signalled"))
            return
        comm.abort()
        q.put((rank, "progress", "aborted after the peer left"))
        launches = ctx.launch_count()
        try:
            comm.sample(cfg, xs, lo, V, u)
            q.put((rank, "error", "the sharded call did not refuse an aborted communicator"))
            return
        except VdxsError as exc:
            code = exc.code
        try:
            comm.status()
            status_code = abi.OK
        except VdxsError as exc:
            status_code = exc.code
        q.put((rank, "ok", {"first": first.tolist(), "code": code, "status": status_code,
                            "launched": ctx.launch_count() - launches}))
        comm.close()
        ctx.close()
    except BaseException as exc:
        q.put((rank, "error", repr(exc)))


def test_peer_leaving_between_steps_is_refused_without_a_launch():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from vindexllm_b200.sampler import ShardComm
    uid = ShardComm.unique_id()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    left = mpc.Event()
    procs = [mpc.Process(target=_leaver_worker, args=(r, 2, uid, q, left)) for r in range(2)]
    for p in procs:
        p.start()
    res, log = {}, []
    import queue
    while len(res) < 2:
        try:
            r, status, info = q.get(timeout=180)
        except queue.Empty:
            break
        if status == "progress":
            log.append((r, info))
        else:
            res[r] = (status, info)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():  # only the processes this test started
            p.kill()
            p.join(timeout=10)
    assert set(res) == {0, 1}, f"ranks that reported: {res}; progress: {log}"
    assert res[1][0] == "left", res[1]
    assert res[0][0] == "ok", res[0]
    info = res[0][1]
    assert info["first"] == res[1][1]  # both ranks drew the same tokens in step 1
    assert info["code"] == abi.E_NCCL and info["status"] == abi.E_NCCL
    assert info["launched"] == 0
