"""testbed/UTest.Sampler.pas restated against the CPU oracle (the checker).

Each test mirrors one Section of TSamplerTest (UTest.Sampler.pas:54-61) with the same
inputs (CVocabSize = 10, :44) and the same checks, run through both restatements of
TVdxSampler: the C++ oracle and the independent pure-Python one."""
import numpy as np
import pytest

from oracle import pyref
from vindexllm_b200.abi import default_config

V = 10  # UTest.Sampler.pas:44


def make(kind, oracle_mod):
    if kind == "cpp":
        return CppWrap(oracle_mod.OracleSampler())
    return PyWrap(pyref.PySampler())


class CppWrap:
    def __init__(self, s):
        self.s = s

    def set_config(self, cfg):
        self.s.set_config(cfg)

    def get_config(self):
        return self.s.get_config().as_dict()

    def process(self, logits):
        return self.s.process(np.array(logits, np.float32))

    def add_to_history(self, t):
        self.s.add_to_history(t)


class PyWrap:
    def __init__(self, s):
        self.s = s

    def set_config(self, cfg):
        self.s.set_config(cfg.as_dict())

    def get_config(self):
        return dict(self.s.cfg)

    def process(self, logits):
        return self.s.process([float(np.float32(v)) for v in logits], len(logits))

    def add_to_history(self, t):
        self.s.add_to_history(t)


KINDS = ["cpp", "py"]


@pytest.mark.parametrize("kind", KINDS)
def test_create_destroy_default_config(kind, oracle_mod):  # :68-92
    s = make(kind, oracle_mod)
    c = s.get_config()
    assert c["temperature"] == 0.0
    assert c["top_k"] == 0
    assert c["top_p"] == 1.0
    assert c["min_p"] == 0.0
    assert c["repeat_penalty"] == 1.0
    assert c["repeat_window"] == 64
    assert c["seed"] == 0


@pytest.mark.parametrize("kind", KINDS)
def test_greedy_argmax(kind, oracle_mod):  # :99-133
    logits = [0.1] * V
    logits[7] = 5.0
    s = make(kind, oracle_mod)
    s.set_config(default_config(temperature=0.0))
    assert s.process(logits) == 7
    logits[7] = 0.1
    logits[2] = 9.9
    assert s.process(logits) == 2


@pytest.mark.parametrize("kind", KINDS)
def test_deterministic_reseed(kind, oracle_mod):  # :141-193
    logits = [i * 0.25 for i in range(V)]
    cfg = default_config(temperature=1.0, seed=42)
    seqs = []
    for _ in range(2):
        s = make(kind, oracle_mod)
        s.set_config(cfg)
        seqs.append([s.process(logits) for _ in range(50)])
    assert seqs[0] == seqs[1]


@pytest.mark.parametrize("kind", KINDS)
def test_topk_bound(kind, oracle_mod):  # :200-248
    logits = [0.0] * V
    for i in (1, 4, 8):
        logits[i] = 10.0
    s = make(kind, oracle_mod)
    s.set_config(default_config(temperature=1.0, top_k=3, seed=42))
    assert all(s.process(logits) in (1, 4, 8) for _ in range(200))


@pytest.mark.parametrize("kind", KINDS)
def test_repeat_penalty(kind, oracle_mod):  # :259-327
    logits = [1.0] * V
    cfg = default_config(temperature=1.0, repeat_penalty=1.0, seed=42)
    s = make(kind, oracle_mod)
    s.set_config(cfg)
    plain = sum(s.process(list(logits)) == 3 for _ in range(200))
    cfg = default_config(temperature=1.0, repeat_penalty=2.0, seed=42)
    s = make(kind, oracle_mod)
    s.set_config(cfg)
    s.add_to_history(3)
    pen = sum(s.process(list(logits)) == 3 for _ in range(200))
    assert pen < plain
    assert plain > 5


def test_both_restatements_agree_on_sections(oracle_mod):
    """The two restatements produce the same draw sequences for the sections' inputs."""
    for cfg, logits, hist in [
        (default_config(temperature=1.0, seed=42), [i * 0.25 for i in range(V)], []),
        (default_config(temperature=1.0, top_k=3, seed=42), [10.0 if i in (1, 4, 8) else 0.0 for i in range(V)], []),
        (default_config(temperature=1.0, repeat_penalty=2.0, seed=42), [1.0] * V, [3]),
    ]:
        a, b = make("cpp", oracle_mod), make("py", oracle_mod)
        a.set_config(cfg)
        b.set_config(cfg)
        for t in hist:
            a.add_to_history(t)
            b.add_to_history(t)
        assert [a.process(list(logits)) for _ in range(200)] == [b.process(list(logits)) for _ in range(200)]
