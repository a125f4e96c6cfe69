"""TEST INFRASTRUCTURE ONLY: an independent pure-Python restatement of TVdxSampler.

Written directly from src/VindexLLM.Sampler.pas (line numbers cited per method) and
kept deliberately literal, including the hand-written mod-2^64 helpers WrapAdd /
WrapMul, so that it cross-checks the C++ oracle (oracle/vdx_oracle.cpp) through a
second, separately written path. Loops are pure Python: use it for small vocabularies
only (tests and the golden fixtures under tests/golden/).

Floating-point convention, shared with the C++ oracle and not pinned by any reference
test: Single operands are evaluated in Double (Python float) and rounded to Single on
every store (``f32``); Exp is the C library double exp (``math.exp``).
"""
from __future__ import annotations

import math
import struct
import time

MASK64 = (1 << 64) - 1
HIGH_UINT64 = MASK64


def f32(v: float) -> float:
    """Round a Python float (double) to the nearest Single, as a store into Single does."""
    return struct.unpack("<f", struct.pack("<f", v))[0]


def bf16_bits_to_f32(b: int) -> float:
    return struct.unpack("<f", struct.pack("<I", (b & 0xFFFF) << 16))[0]


# ---- Sampler.pas:160-190: WrapAdd / WrapMul, restated literally -------------------
def wrap_add(a: int, b: int) -> int:
    if b <= HIGH_UINT64 - a:
        return a + b
    return b - (HIGH_UINT64 - a) - 1


def wrap_mul(a: int, b: int) -> int:
    a_lo, a_hi = a & 0xFFFFFFFF, a >> 32
    b_lo, b_hi = b & 0xFFFFFFFF, b >> 32
    result = a_lo * b_lo
    cross1 = a_lo * b_hi
    cross2 = a_hi * b_lo
    result = wrap_add(result, ((cross1 & 0xFFFFFFFF) << 32) & MASK64)
    result = wrap_add(result, ((cross2 & 0xFFFFFFFF) << 32) & MASK64)
    return result


def rot_left(x: int, k: int) -> int:  # Sampler.pas:203-206
    return ((x << k) | (x >> (64 - k))) & MASK64


def splitmix64(state: int) -> tuple[int, int]:  # Sampler.pas:194-201 -> (new_state, result)
    state = wrap_add(state, 0x9E3779B97F4A7C15)
    r = state
    r = wrap_mul(r ^ (r >> 30), 0xBF58476D1CE4E5B9)
    r = wrap_mul(r ^ (r >> 27), 0x94D049BB133111EB)
    return state, r ^ (r >> 31)


DEFAULT_CONFIG = dict(temperature=0.0, top_k=0, top_p=1.0, min_p=0.0,
                      repeat_penalty=1.0, repeat_window=64, seed=0)  # Sampler.pas:100-109


class PySampler:
    """TVdxSampler (Sampler.pas:37-91) with the reference's observable behaviour."""

    def __init__(self):  # Sampler.pas:111-122
        self.cfg = dict(DEFAULT_CONFIG)
        self.history = [0] * self.cfg["repeat_window"]
        self.hist_pos = 0
        self.hist_count = 0
        self.s = [0, 0, 0, 0]
        self.seed_prng(0)

    # -- PRNG -------------------------------------------------------------------
    def seed_prng(self, seed: int):  # Sampler.pas:224-241
        st = (time.perf_counter_ns() if seed == 0 else seed) & MASK64
        out = []
        for _ in range(4):
            st, r = splitmix64(st)
            out.append(r)
        self.s = out

    def next_uint64(self) -> int:  # Sampler.pas:208-222
        s0, s1, s2, s3 = self.s
        result = wrap_mul(rot_left(wrap_mul(s1, 5), 7), 9)
        t = (s1 << 17) & MASK64
        s2 ^= s0
        s3 ^= s1
        s1 ^= s2
        s0 ^= s3
        s2 ^= t
        s3 = rot_left(s3, 45)
        self.s = [s0, s1, s2, s3]
        return result

    def next_float(self) -> float:  # Sampler.pas:243-248
        return f32((self.next_uint64() >> 40) / 16777216.0)

    # -- config / history ---------------------------------------------------------
    def set_config(self, cfg: dict):  # Sampler.pas:132-150
        seed_changed = cfg["seed"] != self.cfg["seed"]
        self.cfg = dict(cfg)
        want = max(0, self.cfg["repeat_window"])
        if len(self.history) != want:
            self.history = [0] * want
            self.hist_pos = 0
            self.hist_count = 0
        if seed_changed:
            self.seed_prng(self.cfg["seed"])

    def add_to_history(self, token: int):  # Sampler.pas:530-539
        w = self.cfg["repeat_window"]
        if w <= 0:
            return
        self.history[self.hist_pos] = token
        self.hist_pos = (self.hist_pos + 1) % w
        if self.hist_count < w:
            self.hist_count += 1

    def reset_history(self):  # Sampler.pas:541-549
        self.hist_pos = 0
        self.hist_count = 0
        if self.cfg["seed"] > 0:
            self.seed_prng(self.cfg["seed"])

    # -- Process -------------------------------------------------------------------
    def process(self, logits: list, vocab: int, uniform: float | None = None) -> int:
        """Sampler.pas:265-528. Mutates ``logits`` (penalty). If ``uniform`` is given it
        replaces the single NextFloat draw, otherwise the PRNG is used."""
        return process_row(self.cfg, logits, vocab, self.history[: self.hist_count],
                           (lambda: self.next_float()) if uniform is None else (lambda: uniform))


def process_row(cfg: dict, x: list, V: int, history: list, draw) -> int:
    """Faithful Process body on a list of Singles; ``draw()`` yields the uniform."""
    p = f32(cfg["repeat_penalty"])
    # Step 0: repetition penalty, Sampler.pas:285-303.
    if p != 1.0 and len(history) > 0:
        for tok in history:
            if 0 <= tok < V:
                v = x[tok]
                if v > 0.0:
                    x[tok] = f32(v / p)
                elif v < 0.0:
                    x[tok] = f32(v * p)
    temp = f32(cfg["temperature"])
    # Greedy, Sampler.pas:305-322.
    if temp == 0.0:
        best, score = 0, x[0]
        for i in range(1, V):
            if x[i] > score:
                best, score = i, x[i]
        return best
    inv_temp = f32(1.0 / temp)  # :325
    top_k = cfg["top_k"]
    min_p = f32(cfg["min_p"])
    top_p = f32(cfg["top_p"])
    if 0 < top_k < V:
        K = top_k
        buf = [0.0] * K
        idx = [0] * K
        max_logit = x[0]
        min_idx, min_val = 0, f32(-1e30)
        for i in range(V):  # :346-383
            v = x[i]
            if v > max_logit:
                max_logit = v
            if i < K:
                buf[i], idx[i] = v, i
                if i == K - 1:
                    min_idx, min_val = 0, buf[0]
                    for j in range(1, K):
                        if buf[j] < min_val:
                            min_idx, min_val = j, buf[j]
            elif v > min_val:
                buf[min_idx], idx[min_idx] = v, i
                min_idx, min_val = 0, buf[0]
                for j in range(1, K):
                    if buf[j] < min_val:
                        min_idx, min_val = j, buf[j]
        lsum = 0.0
        for i in range(K):  # :386-391
            buf[i] = f32(math.exp((buf[i] - max_logit) * inv_temp))
            lsum += buf[i]
        if min_p > 0.0:  # :394-410
            best = buf[0]
            for i in range(1, K):
                if buf[i] > best:
                    best = buf[i]
            thr = f32(best * min_p)
            lsum = 0.0
            for i in range(K):
                if buf[i] < thr:
                    buf[i] = 0.0
                else:
                    lsum += buf[i]
        if top_p < 1.0:  # :413-445
            for i in range(1, K):
                v, ti = buf[i], idx[i]
                j = i - 1
                while j >= 0 and buf[j] < v:
                    buf[j + 1], idx[j + 1] = buf[j], idx[j]
                    j -= 1
                buf[j + 1], idx[j + 1] = v, ti
            target = top_p * lsum
            cum = 0.0
            lsum = 0.0
            for i in range(K):
                if cum < target and buf[i] > 0.0:
                    cum += buf[i]
                    lsum += buf[i]
                else:
                    buf[i] = 0.0
        t = draw() * lsum  # :448-459
        cum = 0.0
        for i in range(K):
            cum += buf[i]
            if cum > t:
                return idx[i]
        return idx[K - 1]
    # Full softmax path, Sampler.pas:463-527.
    probs = [0.0] * V
    max_logit = f32(x[0] * inv_temp)
    for i in range(V):
        v = f32(x[i] * inv_temp)
        probs[i] = v
        if v > max_logit:
            max_logit = v
    lsum = 0.0
    for i in range(V):
        v = f32(math.exp(probs[i] - max_logit))
        probs[i] = v
        lsum += v
    if min_p > 0.0:
        best = probs[0]
        for i in range(1, V):
            if probs[i] > best:
                best = probs[i]
        thr = f32(best * min_p)
        lsum = 0.0
        for i in range(V):
            if probs[i] < thr:
                probs[i] = 0.0
            else:
                lsum += probs[i]
    t = draw() * lsum
    cum = 0.0
    for i in range(V):
        cum += probs[i]
        if cum > t:
            return i
    return V - 1
