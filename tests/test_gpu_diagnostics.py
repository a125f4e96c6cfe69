"""Status and diagnostics entry points: vdxs_device_status, vdxs_set_stage_events and
vdxs_get_launch_count. None of them changes a token; they report on the kernels."""
import ctypes as C

import pytest

from vindexllm_b200 import synth
from vindexllm_b200._lib import VdxsError, check

pytestmark = pytest.mark.gpu


def _inputs(name, batch):
    import torch
    x = synth.make_logits(name, batch=batch)
    h, c = synth.make_history(name, batch=batch)
    u = torch.as_tensor(synth.make_uniforms(name, 1, batch=batch)[0], device="cuda")
    return x, h, c, u


def test_device_status_clean_after_calls(gpu_ctx):
    x, h, c, u = _inputs("c1", 8)
    for _ in range(3):
        gpu_ctx.sample(synth.sampler_config("c1"), x, u, h, c)
    gpu_ctx.device_status()  # raises VdxsError on a non-zero device error word


@pytest.mark.parametrize("name,batch,per_call", [("c4", 16, 2), ("c1", 16, 3), ("c3", 16, 2), ("c4", 2, 1),
                                                 ("c1", 2, 2)])
def test_launch_count(gpu_ctx, name, batch, per_call):
    """Kernels per call: stream stage 1 + finish (k <= 128, and the wide stream for
    k > 128), one cluster kernel for batches of at most 8; + penalty prep when a history
    is given."""
    x, h, c, u = _inputs(name, batch)
    cfg = synth.sampler_config(name)
    n0 = gpu_ctx.launch_count()
    for _ in range(5):
        gpu_ctx.sample(cfg, x, u, h, c)
    assert gpu_ctx.launch_count() - n0 == 5 * per_call


def test_launch_count_full_path(gpu_ctx):
    x, _, _, u = _inputs("c0", 2)
    cfg = synth.sampler_config("c0", top_k=0)
    n0 = gpu_ctx.launch_count()
    gpu_ctx.sample(cfg, x, u)
    assert gpu_ctx.launch_count() - n0 == 2


def test_stage_events_bracket_the_select_pass(gpu_ctx):
    import torch
    x, h, c, u = _inputs("c4", 64)
    cfg = synth.sampler_config("c4")
    call_b, call_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kb, ke = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gpu_ctx.set_stage_events(kb, ke)
    try:
        call_b.record()
        tok = gpu_ctx.sample(cfg, x, u, h, c)
        call_e.record()
        torch.cuda.synchronize()
    finally:
        gpu_ctx.set_stage_events(None, None)
    k_ms = kb.elapsed_time(ke)
    call_ms = call_b.elapsed_time(call_e)
    assert 0.0 < k_ms <= call_ms
    # the hook does not change the result
    ref = gpu_ctx.sample(cfg, x, u, h, c)
    assert torch.equal(tok, ref)


def test_stage_events_need_both(gpu_ctx):
    import torch
    ev = torch.cuda.Event(enable_timing=True)
    ev.record()
    with pytest.raises(VdxsError):
        check(gpu_ctx.lib.vdxs_set_stage_events(gpu_ctx.handle, C.c_void_p(ev.cuda_event), None), gpu_ctx.handle)
    check(gpu_ctx.lib.vdxs_set_stage_events(gpu_ctx.handle, None, None), gpu_ctx.handle)
