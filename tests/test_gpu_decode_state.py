"""Device-resident decode state (vdxs_device_uniforms, vdxs_device_history_push,
vdxs_decode_step) against the host-side stateful sampler, whose PRNG and history ring
follow TVdxSampler (src/VindexLLM.Sampler.pas:208-248 NextFloat, :530-539 AddToHistory,
:265-528 Process): the same uniforms bit for bit, the same tokens step by step, the
same rings and PRNG states afterwards."""
import numpy as np
import pytest

from vindexllm_b200 import abi
from vindexllm_b200.abi import default_config

pytestmark = pytest.mark.gpu


def _logits(rng, B, V, hot):
    import torch
    x = (rng.normal(size=(B, V)) * 2.0).astype(np.float32)
    x[:, hot] += 6.0  # a few strong ids, so that repeats and the penalty matter
    return torch.as_tensor(x, device="cuda")


def test_device_uniforms_match_nextfloat(gpu_ctx):
    from vindexllm_b200.sampler import TVdxSampler, DeviceDecodeState
    B = 37
    host = TVdxSampler(gpu_ctx, batch=B)  # time-seeded rows: distinct streams
    dev = DeviceDecodeState(B, 0, prng_states=[host.GetPrngState(r) for r in range(B)])
    for _ in range(50):
        u = dev.next_uniforms().cpu().numpy()
        h = np.array([host.NextFloat(r) for r in range(B)], np.float32)
        assert (u.view(np.uint32) == h.view(np.uint32)).all()
    host.close()


@pytest.mark.parametrize("mode", [abi.TIES_FAITHFUL, abi.TIES_CANONICAL])
@pytest.mark.parametrize("temperature", [0.8, 0.0])
def test_decode_step_matches_stateful_sampler(gpu_ctx, mode, temperature):
    import torch
    from vindexllm_b200.sampler import TVdxSampler, DeviceDecodeState
    gpu_ctx.set_tie_mode(mode)
    rng = np.random.default_rng(5)
    B, V, W = 12, 50000, 32
    cfg = default_config(temperature=temperature, top_k=40, top_p=0.9, repeat_penalty=1.3, repeat_window=W)
    host = TVdxSampler(gpu_ctx, batch=B)
    host.SetConfig(cfg)  # seed 0 as at creation: the time-seeded rows are kept
    dev = DeviceDecodeState(B, W, prng_states=[host.GetPrngState(r) for r in range(B)])
    hot = rng.choice(V, size=6, replace=False)
    for _ in range(6):
        x = _logits(rng, B, V, hot)
        th = host.Process(x)
        host.AddToHistoryBatch(th)
        td = dev.step(gpu_ctx, cfg, x).cpu().numpy()
        assert (td == th).all(), f"device {td} host {th}"
    gpu_ctx.device_status()
    hist, pos, cnt = dev.hist.cpu().numpy(), dev.pos.cpu().numpy(), dev.count.cpu().numpy()
    states = dev.prng.cpu().numpy().view(np.uint64)
    for r in range(B):
        ids, c, p = host.GetHistory(r)
        assert (c, p) == (int(cnt[r]), int(pos[r]))
        assert ids == hist[r, :c].tolist()
        assert list(host.GetPrngState(r)) == states[r].tolist()  # greedy steps draw nothing
    host.close()
    gpu_ctx.set_tie_mode(abi.TIES_FAITHFUL)


@pytest.mark.parametrize("temperature", [0.8, 0.0])
def test_decode_step_matches_oracle_samplers(gpu_ctx, oracle_mod, temperature):
    """vdxs_decode_step against the CPU restatement of TVdxSampler, one oracle object per
    row: each step the oracle runs Process (Sampler.pas:265-528, which draws NextFloat
    from its own PRNG) and AddToHistory (:530-539) on the same logits; tokens must agree
    at every step, and the rings and PRNG states afterwards."""
    from vindexllm_b200.sampler import DeviceDecodeState
    gpu_ctx.set_tie_mode(abi.TIES_FAITHFUL)
    rng = np.random.default_rng(23)
    B, V, W = 10, 60000, 24
    cfg = default_config(temperature=temperature, top_k=32, top_p=0.9, repeat_penalty=1.25, repeat_window=W,
                         seed=99)
    states = [[0x243F6A8885A308D3 + 7 * r, 0x13198A2E03707344, 0xA4093822299F31D0 ^ r, 0x082EFA98EC4E6C89]
              for r in range(B)]
    orc = []
    for r in range(B):
        o = oracle_mod.OracleSampler()
        o.set_config(cfg)
        o.set_state(states[r])
        orc.append(o)
    dev = DeviceDecodeState(B, W, prng_states=states)
    hot = rng.choice(V, size=6, replace=False)
    for step in range(8):
        x = _logits(rng, B, V, hot)
        xh = x.cpu().numpy()
        want = []
        for r in range(B):
            t = orc[r].process(np.ascontiguousarray(xh[r]).copy())  # Process mutates its logits
            orc[r].add_to_history(t)
            want.append(t)
        got = dev.step(gpu_ctx, cfg, x).cpu().numpy()
        assert (got == np.array(want)).all(), f"step {step}: device {got} oracle {want}"
    gpu_ctx.device_status()
    hist, pos, cnt = dev.hist.cpu().numpy(), dev.pos.cpu().numpy(), dev.count.cpu().numpy()
    prng = dev.prng.cpu().numpy().view(np.uint64)
    for r in range(B):
        ids, c, p = orc[r].history()
        assert (c, p) == (int(cnt[r]), int(pos[r]))
        assert ids[:c] == hist[r, :c].tolist()
        assert orc[r].get_state() == prng[r].tolist()
        orc[r].close()


def test_history_push_and_stop_flags(gpu_ctx):
    import torch
    from vindexllm_b200.sampler import DeviceDecodeState
    B, W = 5, 3
    dev = DeviceDecodeState(B, W)
    stop = torch.tensor([7, 11], dtype=torch.int32, device="cuda")
    seq = [[1, 7, 3, 4, 5], [2, 2, 11, 4, 6], [9, 8, 3, 1, 0], [4, 4, 4, 4, 4]]
    for toks in seq:
        dev.push(torch.tensor(toks, dtype=torch.int32, device="cuda"), stop_ids=stop)
    torch.cuda.synchronize()
    # ring of window 3 after 4 pushes: slot 0 holds the 4th token, slots 1-2 the 2nd and 3rd
    want = np.array([[s[3][r], s1, s2] for r, (s1, s2) in enumerate(zip(seq[1], seq[2])) for s in [seq]])
    assert (dev.hist.cpu().numpy() == want).all()
    assert dev.count.cpu().tolist() == [3] * B and dev.pos.cpu().tolist() == [1] * B
    assert dev.stopped.cpu().tolist() == [0, 1, 1, 0, 0]


@pytest.mark.parametrize("B", [4, 12])  # cluster path; stream path with the penalty prep
def test_decode_step_replayed_from_a_cuda_graph(gpu_ctx, B):
    """A decode step captured once in a CUDA graph (after a warm-up call, so that the
    context's workspace no longer grows) and replayed four times gives the tokens, rings
    and PRNG states of four eager steps from the same state."""
    import torch
    from vindexllm_b200.sampler import DeviceDecodeState
    gpu_ctx.set_tie_mode(abi.TIES_FAITHFUL)
    rng = np.random.default_rng(17)
    V, W = 40000, 16
    cfg = default_config(temperature=0.9, top_k=40, top_p=0.9, repeat_penalty=1.2, repeat_window=W)
    x = _logits(rng, B, V, rng.choice(V, size=5, replace=False))
    states = [[0x9E3779B97F4A7C15 + r, 0xBF58476D1CE4E5B9, 0x94D049BB133111EB, 7 + 3 * r] for r in range(B)]
    eager = DeviceDecodeState(B, W, prng_states=states)
    want = [eager.step(gpu_ctx, cfg, x).cpu().numpy() for _ in range(4)]
    warm = DeviceDecodeState(B, W, prng_states=states)
    tok = torch.empty(B, dtype=torch.int32, device="cuda")
    warm.step(gpu_ctx, cfg, x, tokens=tok)
    torch.cuda.synchronize()
    graphed = DeviceDecodeState(B, W, prng_states=states)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        graphed.step(gpu_ctx, cfg, x, tokens=tok)
    got = []
    for _ in range(4):
        g.replay()
        got.append(tok.cpu().numpy())
    gpu_ctx.device_status()
    for a, b in zip(got, want):
        assert (a == b).all(), f"graph {a} eager {b}"
    assert (graphed.hist.cpu() == eager.hist.cpu()).all()
    assert (graphed.prng.cpu() == eager.prng.cpu()).all()
    assert (graphed.count.cpu() == eager.count.cpu()).all() and (graphed.pos.cpu() == eager.pos.cpu()).all()
    del g
