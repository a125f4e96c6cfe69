"""Unembedding in front of the sampler (TVdxModel.UnembedToLogits, Model.pas:1258-1271,
with shaders/matvec_q4_0.comp:45-88): the GPU logits equal the oracle's restatement of
the shader bit for bit, and the tokens of vdxs_sample_unembed_q4_0 equal the oracle
sampler's on those logits, in both tie modes."""
import numpy as np
import pytest

from vindexllm_b200 import abi, synth
from vindexllm_b200.abi import default_config
from gpu_helpers import NTHREADS

pytestmark = pytest.mark.gpu


def _weights(ctx, V, H, seed):
    from vindexllm_b200.sampler import Q4Weights
    wq = synth.make_q4_0(V, H, seed=seed, device="cuda")
    return wq, Q4Weights(ctx, wq, H, V)


@pytest.mark.parametrize("H", [64, 96, 1152, 2560, 3840])
@pytest.mark.parametrize("B", [1, 3, 8, 11])
def test_unembed_logits_bit_exact(gpu_ctx, oracle_mod, H, B):
    """Odd block counts (H = 96: the last partials take one term fewer), the hidden sizes
    with specialised kernels (1152: a padded last word, 2560, 3840), batches across the
    8/4/2/1-row launch chunks."""
    import torch
    V = 3001
    wq, w = _weights(gpu_ctx, V, H, seed=H + B)
    x = torch.as_tensor(synth.make_hidden(B, H, seed=B), device="cuda")
    got = w.unembed(x).cpu().numpy()
    want = oracle_mod.matvec_q4_0(wq.cpu().numpy(), x.cpu().numpy(), nthreads=NTHREADS)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    w.close()


def test_unembed_special_scales(gpu_ctx, oracle_mod):
    """fp16 scales that are subnormal, negative, zero or large: the dequantised weights stay
    exact and the sums bit-exact."""
    import torch
    V, H = 512, 256
    wq = synth.make_q4_0(V, H, seed=3, device="cuda").view(V, H // 32, 18)
    special = torch.tensor([0x0001, 0x03FF, 0x8001, 0x0000, 0x8000, 0x7BFF, 0xFBFF, 0x3C00], dtype=torch.int32)
    sc = special[torch.arange(V * (H // 32)) % len(special)].to(torch.int16).view(V, H // 32)
    wq[:, :, 0:2] = sc.view(torch.uint8).reshape(V, H // 32, 2).cuda()
    wq = wq.reshape(V, -1).contiguous()
    from vindexllm_b200.sampler import Q4Weights
    w = Q4Weights(gpu_ctx, wq, H, V)
    x = torch.as_tensor(synth.make_hidden(2, H, seed=9) * 1e-3, device="cuda")
    got = w.unembed(x).cpu().numpy()
    want = oracle_mod.matvec_q4_0(wq.cpu().numpy(), x.cpu().numpy(), nthreads=NTHREADS)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    w.close()


@pytest.mark.parametrize("mode", [abi.TIES_FAITHFUL, abi.TIES_CANONICAL])
def test_sample_unembed_full_size(gpu_ctx, oracle_mod, mode):
    """Gemma-3 sized tied embedding (262144 x 2560, Q4_0): logits bit-exact for 2 rows and
    tokens equal to the oracle sampler on the oracle's logits, with the c0 and c1
    sampling configurations (penalty history included)."""
    import torch
    V, H, B = synth.VOCAB, synth.HIDDEN, 2
    wq, w = _weights(gpu_ctx, V, H, seed=7000)
    x = torch.as_tensor(synth.make_hidden(B, H), device="cuda")
    want = oracle_mod.matvec_q4_0(wq.cpu().numpy(), x.cpu().numpy(), nthreads=NTHREADS)
    got = w.unembed(x).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    gpu_ctx.set_tie_mode(mode)
    rng = np.random.default_rng(1)
    for name in ("c0", "c1"):
        cfg = synth.sampler_config(name)
        u = rng.random(B).astype(np.float32)
        hist = rng.integers(0, V, size=(B, 64)).astype(np.int32)
        cnt = np.full(B, 64, np.int32)
        tok = w.sample(cfg, x, torch.as_tensor(u, device="cuda"), torch.as_tensor(hist, device="cuda"),
                       torch.as_tensor(cnt, device="cuda")).cpu().numpy()
        ot = oracle_mod.sample_batch(cfg, want, u, hist, cnt, mode, nthreads=NTHREADS)[0]
        assert (tok == ot).all(), f"{name}: gpu {tok} oracle {ot}"
    w.close()


def test_unembed_rejects_bad_shapes(gpu_ctx):
    import ctypes as C
    import torch
    from vindexllm_b200 import _lib
    lib = _lib.load()
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    h = C.c_void_p()
    rc = lib.vdxs_q4_0_prepare(gpu_ctx.handle, C.c_void_p(buf.data_ptr()), 100, 10, None, C.byref(h))
    assert rc == abi.E_INVALID_ARG and not h.value
    rc = lib.vdxs_q4_0_prepare(gpu_ctx.handle, None, 64, 10, None, C.byref(h))
    assert rc == abi.E_INVALID_ARG
