"""Seeded synthetic inputs for the five benchmark configurations.

The reference publishes no dataset for this path; these generators reproduce the
shapes and value distributions named by the benchmark configurations:

  c0  B=1    V=262144 fp32  4*N(0,1), +12 on 8 seeded indices   T=1.0 k=64   p=0.95
  c1  B=64   V=262144 fp32  as c0, per-row seeds; 512-id history, penalty 1.1
                                                                 T=0.7 k=40   p=0.9
  c2  B=256  V=262144 bf16  3*N(0,1) + 10*r^-1.1 over a seeded permutation of ranks
                                                                 T=1.0 k=64   p=0.95
  c3  B=1024 V=262144 fp32  0.5*N(0,1), 1% of entries set to the row's k-th largest
                            value (ties straddle the top-k boundary)  T=1.3 k=1024 p=0.99
  c4  B=512  V=262144 fp32  as c2 in fp32; contiguous vocab shards   T=1.0 k=64   p=0.95

Uniforms are what TVdxSampler.NextFloat returns (src/VindexLLM.Sampler.pas:243-248):
(xoshiro256** >> 40) / 2^24 from one SplitMix64-seeded stream per row.
"""
from __future__ import annotations

import numpy as np

from .abi import VdxsConfig, default_config

VOCAB = 262144

CONFIGS = {
    "c0": dict(batch=1, dtype="f32", kind="peaks", temperature=1.0, top_k=64, top_p=0.95,
               repeat_penalty=1.0, window=0),
    "c1": dict(batch=64, dtype="f32", kind="peaks", temperature=0.7, top_k=40, top_p=0.9,
               repeat_penalty=1.1, window=512),
    "c2": dict(batch=256, dtype="bf16", kind="zipf", temperature=1.0, top_k=64, top_p=0.95,
               repeat_penalty=1.0, window=0),
    "c3": dict(batch=1024, dtype="f32", kind="flat_ties", temperature=1.3, top_k=1024, top_p=0.99,
               repeat_penalty=1.0, window=0),
    "c4": dict(batch=512, dtype="f32", kind="zipf", temperature=1.0, top_k=64, top_p=0.95,
               repeat_penalty=1.0, window=0),
}

_SEED_BASE = {"c0": 1000, "c1": 2000, "c2": 3000, "c3": 4000, "c4": 5000}


def sampler_config(name: str, **overrides) -> VdxsConfig:
    c = CONFIGS[name]
    d = dict(temperature=c["temperature"], top_k=c["top_k"], top_p=c["top_p"], min_p=0.0,
             repeat_penalty=c["repeat_penalty"], repeat_window=c["window"] or 64, seed=42)
    d.update(overrides)
    return default_config(**d)


def make_logits(name: str, step: int = 0, batch: int | None = None, vocab: int = VOCAB,
                device: str = "cuda", dtype: str | None = None, kind: str | None = None):
    """[batch, vocab] logits as a torch tensor (float32 or bfloat16) on ``device``."""
    import torch
    c = CONFIGS[name]
    B = c["batch"] if batch is None else batch
    kind = kind or c["kind"]
    dtype = dtype or c["dtype"]
    g = torch.Generator(device=device)
    g.manual_seed(_SEED_BASE[name] * 100003 + step)
    if kind == "peaks":
        x = torch.randn(B, vocab, generator=g, device=device, dtype=torch.float32) * 4.0
        peaks = torch.rand(B, vocab, generator=g, device=device).topk(min(8, vocab), dim=1).indices
        x.scatter_add_(1, peaks, torch.full(peaks.shape, 12.0, device=device))
    elif kind == "zipf":
        x = torch.randn(B, vocab, generator=g, device=device, dtype=torch.float32) * 3.0
        ranks = torch.arange(1, vocab + 1, device=device, dtype=torch.float64)
        bonus = (10.0 * ranks.pow(-1.1)).to(torch.float32).expand(B, vocab)
        if str(device).startswith("cuda"):
            perm = torch.rand(B, vocab, generator=g, device=device).argsort(dim=1)
        else:  # row-wise randperm is much cheaper than a batched argsort on the host
            perm = torch.stack([torch.randperm(vocab, generator=g) for _ in range(B)])
        x.scatter_add_(1, perm, bonus.contiguous())
    elif kind == "flat_ties":
        x = torch.randn(B, vocab, generator=g, device=device, dtype=torch.float32) * 0.5
        k = min(c["top_k"], vocab)
        kth = x.topk(k, dim=1).values[:, -1:]
        mask = torch.rand(B, vocab, generator=g, device=device) < 0.01
        x = torch.where(mask, kth.expand(B, vocab), x)
    else:
        raise ValueError(kind)
    if dtype == "bf16":
        return x.to(torch.bfloat16).contiguous()
    return x.contiguous()


def make_history(name: str, step: int = 0, batch: int | None = None, vocab: int = VOCAB,
                 device: str = "cuda"):
    """[batch, window] int32 history ids (uniform in [0, vocab), duplicates allowed) and
    [batch] counts, or (None, None) for configurations without a penalty."""
    import torch
    c = CONFIGS[name]
    if not c["window"]:
        return None, None
    B = c["batch"] if batch is None else batch
    g = torch.Generator(device=device)
    g.manual_seed(_SEED_BASE[name] * 100003 + 50000 + step)
    h = torch.randint(0, vocab, (B, c["window"]), generator=g, device=device, dtype=torch.int64)
    return h.to(torch.int32).contiguous(), torch.full((B,), c["window"], dtype=torch.int32, device=device)


# ---- xoshiro256** uniforms (Sampler.pas:157-248), vectorised over rows -------------
_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(state):
    state = state + np.uint64(0x9E3779B97F4A7C15)
    z = state
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return state, z ^ (z >> np.uint64(31))


def _rotl(x, k):
    return (x << np.uint64(k)) | (x >> np.uint64(64 - k))


def uniform_streams(seeds: np.ndarray, n: int) -> np.ndarray:
    """[n, len(seeds)] NextFloat values: row r of the batch uses SeedPRNG(seeds[r])."""
    with np.errstate(over="ignore"):
        st = np.asarray(seeds, dtype=np.uint64).copy()
        s = []
        for _ in range(4):
            st, z = _splitmix64(st)
            s.append(z)
        s0, s1, s2, s3 = s
        out = np.empty((n, len(st)), np.float32)
        for i in range(n):
            res = _rotl(s1 * np.uint64(5), 7) * np.uint64(9)
            t = s1 << np.uint64(17)
            s2 ^= s0
            s3 ^= s1
            s1 ^= s2
            s0 ^= s3
            s2 ^= t
            s3 = _rotl(s3, 45)
            out[i] = ((res >> np.uint64(40)).astype(np.float64) / 16777216.0).astype(np.float32)
    return out


def make_uniforms(name: str, steps: int, batch: int | None = None) -> np.ndarray:
    """[steps, batch] uniforms: row r is the NextFloat stream of SeedPRNG(base + r)."""
    B = CONFIGS[name]["batch"] if batch is None else batch
    seeds = np.arange(B, dtype=np.uint64) + np.uint64(_SEED_BASE[name] * 7 + 1)
    return uniform_streams(seeds, steps)


# Unembedding inputs (TVdxModel.UnembedToLogits, Model.pas:1258-1271): a tied Gemma-3
# sized embedding (262144 x 2560) in Q4_0 and normed hidden vectors. No checkpoint is
# available, so the blocks are seeded: fp16 scales ~ |N(0, 0.02)|, uniform nibbles.
HIDDEN = 2560


def make_q4_0(vocab: int = VOCAB, hidden: int = HIDDEN, seed: int = 7000, device: str = "cuda"):
    """[vocab, hidden / 32 * 18] uint8 Q4_0 blocks as a torch tensor on ``device`` (seeded
    per device): fp16 scale, then 16 bytes whose low nibbles are elements 0..15 and high
    nibbles elements 16..31 of the block."""
    import torch
    assert hidden % 32 == 0
    g = torch.Generator(device=device).manual_seed(seed)
    nb = hidden // 32
    out = torch.randint(0, 256, (vocab, nb, 18), dtype=torch.uint8, device=device, generator=g)
    scales = (torch.randn((vocab, nb), device=device, generator=g).abs() * 0.02).to(torch.float16)
    out[:, :, 0:2] = scales.view(torch.uint8).reshape(vocab, nb, 2)
    return out.reshape(vocab, nb * 18)


def make_hidden(batch: int, hidden: int = HIDDEN, seed: int = 7100) -> np.ndarray:
    """[batch, hidden] float32 hidden vectors (RMS-normed scale: ~N(0, 1) entries)."""
    return np.random.default_rng(seed).normal(size=(batch, hidden)).astype(np.float32)
