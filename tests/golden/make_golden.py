"""Generates tests/golden/sampler_cases.json from oracle/pyref.py, the pure-Python
restatement of TVdxSampler.Process (src/VindexLLM.Sampler.pas:265-528).

The reference ships no numeric vectors (it is Delphi; no compiler exists here), so the
fixtures are produced by the restatement that is independent of the C++ oracle and of
the CUDA library; tests check both against them. Run: python tests/golden/make_golden.py
"""
import json
import os
import struct
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import pyref  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sampler_cases.json")


def bits(a):
    return [struct.unpack("<I", struct.pack("<f", float(v)))[0] for v in a]


def case(cfg, logits, history, u):
    x = [float(np.float32(v)) for v in logits]
    tok = pyref.process_row(cfg, list(x), len(x), list(history), lambda: u)
    return dict(cfg=cfg, logits_bits=bits(x), history=[int(h) for h in history],
                uniform_bits=bits([u])[0], token=int(tok))


def main():
    rng = np.random.default_rng(20261201)
    cases = []
    base = dict(temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, repeat_penalty=1.0, repeat_window=64, seed=0)
    # UTest.Sampler.pas inputs with explicit uniforms.
    sec = [
        (dict(base, temperature=0.0), [5.0 if i == 7 else 0.1 for i in range(10)], []),
        (dict(base, temperature=0.0), [9.9 if i == 2 else 0.1 for i in range(10)], []),
        (dict(base), [i * 0.25 for i in range(10)], []),
        (dict(base, top_k=3), [10.0 if i in (1, 4, 8) else 0.0 for i in range(10)], []),
        (dict(base, repeat_penalty=2.0), [1.0] * 10, [3]),
    ]
    for cfg, lg, h in sec:
        for u in (0.0, 0.1, 0.3333333, 0.5, 0.9, 0.99999994):
            cases.append(case(cfg, lg, h, float(np.float32(u))))
    # Branch coverage on small vocabularies, with ties and penalties.
    temps = [0.0, 0.3, 0.7, 1.0, 1.3, 2.0]
    for n in range(400):
        V = int(rng.integers(1, 200))
        style = n % 4
        if style == 0:
            x = rng.normal(size=V) * 3
        elif style == 1:
            x = np.round(rng.normal(size=V) * 2) / 2  # heavy ties
        elif style == 2:
            x = np.float32(rng.normal(size=V) * 4).astype(np.float32)
            x = (x.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)  # bf16-representable
        else:
            x = rng.normal(size=V) * 0.2
            x[rng.integers(0, V, size=max(1, V // 10))] = 1.5
        top_k = int(rng.choice([0, 1, 2, 3, 5, 16, max(1, V - 1), V, V + 3]))
        cfg = dict(base, temperature=float(np.float32(rng.choice(temps))), top_k=top_k,
                   top_p=float(np.float32(rng.choice([1.0, 0.99, 0.9, 0.5, 0.1, 0.0]))),
                   min_p=float(np.float32(rng.choice([0.0, 0.0, 0.05, 0.3]))),
                   repeat_penalty=float(np.float32(rng.choice([1.0, 1.0, 1.1, 2.0, 0.8]))))
        hist = list(rng.integers(-3, V + 3, size=int(rng.integers(0, 12))))
        if hist and rng.random() < 0.5:
            hist += [hist[0]] * 3  # duplicates compound
        u = float(np.float32(int(rng.integers(0, 1 << 24)) / 16777216.0))
        cases.append(case(cfg, x, hist, u))
    with open(OUT, "w") as f:
        json.dump({"generator": "oracle/pyref.py", "cases": cases}, f, separators=(",", ":"))
    print(f"wrote {len(cases)} cases to {OUT}")


if __name__ == "__main__":
    main()
