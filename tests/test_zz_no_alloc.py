"""vdxs_sample_noalloc: the allocation-free entry point, for callers that cannot allocate
device memory while sampling (a host that reserves all GPU memory at model load and
forbids later allocations, or a decode loop that cannot take cudaMalloc's device-wide
synchronisation). It must return the same tokens as vdxs_sample, call after call, while
sharing one fixed device array; vdxs_noalloc_status reports its device error word
without a context. This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

from vindexllm_b200 import _lib, abi, synth

pytestmark = pytest.mark.gpu


def _noalloc(lib, cfg, mode, x, u, h, c, tok=None):
    import torch
    if tok is None:
        tok = torch.full((x.shape[0],), -7, dtype=torch.int32, device=x.device)
    hs = h.shape[1] if h is not None else 1
    rc = lib.vdxs_sample_noalloc(C.byref(cfg), mode, C.c_void_p(x.data_ptr()),
                                 abi.DTYPE_BF16 if x.dtype == torch.bfloat16 else abi.DTYPE_F32,
                                 x.shape[0], x.shape[1], x.stride(0),
                                 None if h is None else C.c_void_p(h.data_ptr()), hs,
                                 None if c is None else C.c_void_p(c.data_ptr()), C.c_void_p(u.data_ptr()),
                                 C.c_void_p(tok.data_ptr()), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == abi.OK, lib.vdxs_last_error(None)
    rc = lib.vdxs_noalloc_status(C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == abi.OK, lib.vdxs_last_error(None)
    return tok.cpu().numpy()


def _inputs(name, step, batch):
    import torch
    x = synth.make_logits(name, step=step, batch=batch)
    h, c = synth.make_history(name, step=step, batch=batch)
    u = torch.as_tensor(synth.make_uniforms(name, step + 1, batch=x.shape[0])[step], device="cuda")
    return x, h, c, u


@pytest.mark.parametrize("name,batch", [("c4", None), ("c1", None), ("c2", 64), ("c0", None)])
def test_noalloc_matches_context_entry(name, batch):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from vindexllm_b200.sampler import SamplerContext
    lib = _lib.load()
    cfg = synth.sampler_config(name)
    ctx = SamplerContext(0)
    for mode in (abi.TIES_FAITHFUL, abi.TIES_CANONICAL):
        ctx.set_tie_mode(mode)
        for step in range(2):  # two calls in a row share and reuse the fixed array
            x, h, c, u = _inputs(name, step, batch)
            want = ctx.sample(cfg, x, u, h, c).cpu().numpy()
            got = _noalloc(lib, cfg, mode, x, u, h, c)
            assert (got == want).all(), f"{name} step {step} mode {mode}"
    ctx.close()


def test_noalloc_leaves_device_memory_unchanged():
    """Once the kernels are loaded (the first calls), further calls change the device's
    free memory by nothing: no allocation of any size."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = _lib.load()
    cfg = synth.sampler_config("c4")
    x, h, c, u = _inputs("c4", 0, 128)
    tok = torch.empty(x.shape[0], dtype=torch.int32, device="cuda")
    first = _noalloc(lib, cfg, abi.TIES_FAITHFUL, x, u, h, c, tok)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        got = _noalloc(lib, cfg, abi.TIES_FAITHFUL, x, u, h, c, tok)
        assert (got == first).all()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes"


def _fresh_process_worker(q):
    """Runs in a new process: the allocation-free call is the first library call, with no
    context anywhere in the process."""
    try:
        import torch
        torch.cuda.set_device(0)
        lib = _lib.load()
        out = []
        for name in ("c4", "c1"):
            cfg = synth.sampler_config(name)
            x, h, c, u = _inputs(name, 0, 64)
            out.append(_noalloc(lib, cfg, abi.TIES_FAITHFUL, x, u, h, c))
        q.put(("ok", out))
    except BaseException as exc:  # report to the parent instead of hanging it
        q.put(("error", repr(exc)))


def test_noalloc_first_call_in_a_fresh_process():
    import torch
    import torch.multiprocessing as mp
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_fresh_process_worker, args=(q,))
    p.start()
    status, res = q.get(timeout=300)
    p.join(timeout=60)
    assert status == "ok", res
    from vindexllm_b200.sampler import SamplerContext
    sc = SamplerContext(0)
    for name, got in zip(("c4", "c1"), res):
        x, h, c, u = _inputs(name, 0, 64)
        want = sc.sample(synth.sampler_config(name), x, u, h, c).cpu().numpy()
        assert (got == want).all(), name
    sc.close()


def test_noalloc_rejects_oversized_requests():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = _lib.load()
    cfg = synth.sampler_config("c3")  # batch 1024, top_k 1024: workspace beyond the fixed array
    x = torch.zeros((1024, 262144), dtype=torch.float32, device="cuda")
    u = torch.zeros(1024, dtype=torch.float32, device="cuda")
    tok = torch.empty(1024, dtype=torch.int32, device="cuda")
    rc = lib.vdxs_sample_noalloc(C.byref(cfg), abi.TIES_FAITHFUL, C.c_void_p(x.data_ptr()), abi.DTYPE_F32,
                                 1024, 262144, 262144, None, 1, None, C.c_void_p(u.data_ptr()),
                                 C.c_void_p(tok.data_ptr()), None)
    assert rc == abi.E_UNSUPPORTED
    assert b"allocation-free" in lib.vdxs_last_error(None)


def test_noalloc_large_top_k():
    """top_k above 1024 (the large top-k kernel) takes its per-CTA workspace from the same
    fixed array: rows of c4 with K = 65536 (1.5 MiB per CTA, whole-row select) and K = 2000
    (stage-1 row lists first) give the context entry's tokens."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from vindexllm_b200.sampler import SamplerContext
    lib = _lib.load()
    ctx = SamplerContext(0)
    for top_k in (65536, 2000):
        cfg = synth.sampler_config("c4", top_k=top_k)
        for mode in (abi.TIES_FAITHFUL, abi.TIES_CANONICAL):
            ctx.set_tie_mode(mode)
            x, h, c, u = _inputs("c4", 0, 2)
            want = ctx.sample(cfg, x, u, h, c).cpu().numpy()
            got = _noalloc(lib, cfg, mode, x, u, h, c)
            assert (got == want).all(), f"top_k {top_k} mode {mode}"
    ctx.close()


def test_noalloc_small_batch_wide_topk():
    """Batch 64 with top_k 1024: the context entry sizes the row lists for 37 stage-1 warps
    per row (about 116 MB); the fixed array takes the shorter lists, whose overflowing rows
    are selected from the whole row. Both give the same tokens."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from vindexllm_b200.sampler import SamplerContext
    lib = _lib.load()
    ctx = SamplerContext(0)
    cfg = synth.sampler_config("c4", top_k=1024)
    for mode in (abi.TIES_FAITHFUL, abi.TIES_CANONICAL):
        ctx.set_tie_mode(mode)
        x, h, c, u = _inputs("c4", 0, 64)
        want = ctx.sample(cfg, x, u, h, c).cpu().numpy()
        got = _noalloc(lib, cfg, mode, x, u, h, c)
        assert (got == want).all(), f"mode {mode}"
    ctx.close()
