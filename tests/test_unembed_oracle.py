"""The oracle's unembedding (oracle/vdx_oracle.cpp, vdxo_matvec_q4_0) against an
independent numpy restatement of shaders/matvec_q4_0.comp:45-88: 64 float32 partial sums
(partial t takes elements t, t + 64, ... in order, acc += (qval * scale) * x with each
operation rounded), then the pairwise tree over strides 32..1. numpy float32 arithmetic
rounds every operation, so the two must agree bit for bit."""
import numpy as np
import pytest


def _q4_0(rng, V, H):
    nb = H // 32
    w = rng.integers(0, 256, size=(V, nb, 18), dtype=np.uint8)
    scales = (np.abs(rng.normal(size=(V, nb))) * 0.05).astype(np.float16)
    scales.flat[::7] = np.float16(-0.0)
    scales.flat[3::11] = np.float16(6.0e-8)  # subnormal
    w[:, :, 0:2] = scales.view(np.uint8).reshape(V, nb, 2)
    return w.reshape(V, nb * 18)


def _shader_numpy(w, x):
    V = w.shape[0]
    H = x.shape[0]
    nb = H // 32
    blk = w.reshape(V, nb, 18)
    scale = blk[:, :, 0:2].copy().view(np.float16).reshape(V, nb).astype(np.float32)
    qs = blk[:, :, 2:]
    lo = (qs & 15).astype(np.int32)
    hi = (qs >> 4).astype(np.int32)
    nib = np.concatenate([lo, hi], axis=2).reshape(V, H)  # element 32j + i
    qval = (nib - 8).astype(np.float32)
    deq = qval * np.repeat(scale, 32, axis=1)  # exact products
    partial = np.zeros((V, 64), np.float32)
    for tid in range(64):
        acc = np.zeros(V, np.float32)
        for elem in range(tid, H, 64):
            acc = acc + deq[:, elem] * x[elem]
        partial[:, tid] = acc
    stride = 32
    while stride > 0:
        partial[:, :stride] = partial[:, :stride] + partial[:, stride:2 * stride]
        stride //= 2
    return partial[:, 0]


@pytest.mark.parametrize("H", [32, 64, 96, 256])
def test_oracle_matvec_matches_numpy_shader(H):
    from oracle import oracle
    oracle.build()
    rng = np.random.default_rng(H)
    V = 300
    w = _q4_0(rng, V, H)
    x = rng.normal(size=(2, H)).astype(np.float32)
    got = oracle.matvec_q4_0(w, x, nthreads=2)
    for b in range(2):
        want = _shader_numpy(w, x[b])
        assert np.array_equal(got[b].view(np.uint32), want.view(np.uint32)), f"H={H} row {b}"
