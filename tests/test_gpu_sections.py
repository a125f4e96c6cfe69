"""testbed/UTest.Sampler.pas through the GPU library's TVdxSampler mirror.

Same sections and checks as the reference (UTest.Sampler.pas:54-61, CVocabSize=10), plus
a draw-for-draw comparison with the oracle's TVdxSampler under the same seed."""
import numpy as np
import pytest

from vindexllm_b200.abi import default_config
from vindexllm_b200.sampler import TVdxSampler

pytestmark = pytest.mark.gpu
V = 10


@pytest.fixture(autouse=True)
def faithful_mode(gpu_ctx):
    """TVdxSampler semantics: the context must be in FAITHFUL mode (the default)."""
    from vindexllm_b200 import abi
    gpu_ctx.set_tie_mode(abi.TIES_FAITHFUL)


def dev(a):
    import torch
    return torch.as_tensor(np.asarray(a, np.float32), device="cuda")[None, :]


def test_create_destroy_default_config(gpu_ctx):  # :68-92
    s = TVdxSampler(gpu_ctx)
    c = s.GetConfig()
    assert (c.temperature, c.top_k, c.top_p, c.min_p, c.repeat_penalty, c.repeat_window, c.seed) == \
        (0.0, 0, 1.0, 0.0, 1.0, 64, 0)
    s.close()


def test_greedy_argmax(gpu_ctx):  # :99-133
    logits = [0.1] * V
    logits[7] = 5.0
    s = TVdxSampler(gpu_ctx)
    s.SetConfig(TVdxSampler.DefaultConfig(temperature=0.0))
    assert s.Process(dev(logits)) == 7
    logits[7] = 0.1
    logits[2] = 9.9
    assert s.Process(dev(logits)) == 2


def test_deterministic_reseed(gpu_ctx, oracle_mod):  # :141-193
    logits = [i * 0.25 for i in range(V)]
    cfg = default_config(temperature=1.0, seed=42)
    seqs = []
    for _ in range(2):
        s = TVdxSampler(gpu_ctx)
        s.SetConfig(cfg)
        seqs.append([s.Process(dev(logits)) for _ in range(50)])
    assert seqs[0] == seqs[1]
    o = oracle_mod.OracleSampler()
    o.set_config(cfg)
    assert seqs[0] == [o.process(np.array(logits, np.float32)) for _ in range(50)]


def test_topk_bound(gpu_ctx, oracle_mod):  # :200-248
    logits = [10.0 if i in (1, 4, 8) else 0.0 for i in range(V)]
    cfg = default_config(temperature=1.0, top_k=3, seed=42)
    s = TVdxSampler(gpu_ctx)
    s.SetConfig(cfg)
    got = [s.Process(dev(logits)) for _ in range(200)]
    assert all(t in (1, 4, 8) for t in got)
    o = oracle_mod.OracleSampler()
    o.set_config(cfg)
    # top_p = 1: the reference walks its min-buffer slot order; faithful mode matches it.
    assert got == [o.process(np.array(logits, np.float32)) for _ in range(200)]


def test_repeat_penalty(gpu_ctx, oracle_mod):  # :259-327
    logits = [1.0] * V
    s = TVdxSampler(gpu_ctx)
    s.SetConfig(default_config(temperature=1.0, repeat_penalty=1.0, seed=42))
    plain = sum(s.Process(dev(logits)) == 3 for _ in range(200))
    s = TVdxSampler(gpu_ctx)
    cfg = default_config(temperature=1.0, repeat_penalty=2.0, seed=42)
    s.SetConfig(cfg)
    s.AddToHistory(3)
    got = [s.Process(dev(logits)) for _ in range(200)]
    assert sum(t == 3 for t in got) < plain and plain > 5
    o = oracle_mod.OracleSampler()
    o.set_config(cfg)
    o.add_to_history(3)
    assert got == [o.process(np.array(logits, np.float32)) for _ in range(200)]


def test_host_logits_process_and_history(gpu_ctx, oracle_mod):
    """Process(PSingle, V) with host logits, a batch of rows, history ring wrap-around."""
    rng = np.random.default_rng(5)
    B, Vb = 4, 5000
    cfg = default_config(temperature=0.8, top_k=20, top_p=0.9, repeat_penalty=1.3, repeat_window=8, seed=7)
    s = TVdxSampler(gpu_ctx, batch=B)
    s.SetConfig(cfg)
    objs = []
    for r in range(B):
        o = oracle_mod.OracleSampler()
        o.set_config(cfg)
        objs.append(o)
    for step in range(30):
        x = (rng.normal(size=(B, Vb)) * 2).astype(np.float32)
        got = s.Process(x)
        want = [objs[r].process(x[r].copy()) for r in range(B)]
        assert list(got) == want, step
        s.AddToHistoryBatch(got)
        for r in range(B):
            objs[r].add_to_history(int(got[r]))
    ids, cnt, pos = s.GetHistory(1)
    oi, oc, op = objs[1].history()
    assert (ids, cnt, pos) == (oi[:cnt], oc, op)
    s.ResetHistory()
    assert s.GetHistory(0)[1] == 0


def test_prng_state_roundtrip(gpu_ctx, oracle_mod):
    s = TVdxSampler(gpu_ctx)
    s.SetConfig(default_config(seed=1234))
    o = oracle_mod.OracleSampler()
    o.set_config(default_config(seed=1234))
    assert s.GetPrngState() == o.get_state()
    assert [s.NextFloat() for _ in range(10)] == [o.next_float() for _ in range(10)]
    st = s.GetPrngState()
    a = [s.NextFloat() for _ in range(5)]
    s.SetPrngState(st)
    assert [s.NextFloat() for _ in range(5)] == a
