"""top_k above 1024 (the reference accepts any 0 < TopK < V, Sampler.pas:327): the large
top-k kernel against the CPU oracle, token ids and flags bit-exact in both tie modes, at
K = 2000, 65536 and V - 1 for fp32 and bf16 rows, with penalties, min-p, top-p below and
at 1 (slot-order walks), ties at the boundary, and a planted top-p cut that lands exactly
on a partial sum."""
import numpy as np
import pytest

from vindexllm_b200 import abi
from vindexllm_b200.abi import default_config
from gpu_helpers import gpu_run, oracle_run, compare, to_host_bits

pytestmark = pytest.mark.gpu

MODES = [abi.TIES_FAITHFUL, abi.TIES_CANONICAL]


def _t(a, dtype=None):
    import torch
    return torch.as_tensor(a, device="cuda", dtype=dtype)


def _check(ctx, oracle_mod, cfg, x, u, hist=None, cnt=None, mode=abi.TIES_FAITHFUL, out_k=16, label=""):
    """x: a torch CUDA tensor (fp32 or bf16)."""
    g = gpu_run(ctx, cfg, x, u, None if hist is None else _t(hist), None if cnt is None else _t(cnt), mode,
                out_k=out_k)
    o = oracle_run(oracle_mod, cfg, to_host_bits(x), u, hist, cnt, mode, out_k=out_k)
    compare(g, o, mode, label=label)
    return g, o


@pytest.mark.parametrize("mode", MODES)
def test_large_topk_random_small_vocab(gpu_ctx, oracle_mod, mode):
    """Many configurations on small rows: every K in (1024, V), both dtypes."""
    import torch
    rng = np.random.default_rng(41)
    for trial in range(10):
        B = int(rng.integers(1, 20))
        V = int(rng.choice([1500, 3000, 5001]))
        K = int(rng.choice([1025, 1200, V // 2, V - 2, V - 1]))
        x = rng.normal(size=(B, V)) * float(rng.choice([0.5, 3.0]))
        if trial % 3 == 0:
            x = np.round(x * 4) / 4  # many ties
        x = x.astype(np.float32)
        cfg = default_config(temperature=float(rng.choice([0.6, 1.0, 1.8])), top_k=K,
                             top_p=float(rng.choice([1.0, 0.95, 0.5])), min_p=float(rng.choice([0.0, 0.05])),
                             repeat_penalty=float(rng.choice([1.0, 1.3])))
        hist = rng.integers(-2, V + 2, size=(B, 32)).astype(np.int32)
        cnt = rng.integers(0, 33, size=B).astype(np.int32)
        u = rng.random(B).astype(np.float32)
        xt = _t(x)
        if trial % 2:
            xt = xt.to(torch.bfloat16)
        _check(gpu_ctx, oracle_mod, cfg, xt, u, hist, cnt, mode, out_k=min(K, 64),
               label=f"trial{trial} B{B} V{V} K{K} bf16{trial % 2} {cfg.as_dict()}")


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("K", [2000, 65536, 262143])
def test_large_topk_full_vocab(gpu_ctx, oracle_mod, mode, dtype, K):
    """V = 262144 rows (c4's vocabulary): K = 2000, 65536 and V - 1, with top-p below 1,
    at 1 (the reference walks slot order), and a repetition penalty."""
    import torch
    V = 262144
    B = 3 if K == 2000 else 2
    rng = np.random.default_rng(K + (7 if dtype == "bf16" else 0))
    x = (rng.normal(size=(B, V)) * 2.0).astype(np.float32)
    xt = _t(x)
    if dtype == "bf16":
        xt = xt.to(torch.bfloat16)
    hist = rng.integers(0, V, size=(B, 64)).astype(np.int32)
    cnt = np.full(B, 64, np.int32)
    u = rng.random(B).astype(np.float32)
    for cfg in [default_config(temperature=1.0, top_k=K, top_p=0.9, repeat_penalty=1.2),
                default_config(temperature=0.8, top_k=K, top_p=1.0, min_p=0.01)]:
        _check(gpu_ctx, oracle_mod, cfg, xt, u, hist, cnt, mode, label=f"K{K} {dtype} {cfg.as_dict()}")


@pytest.mark.parametrize("mode", MODES)
def test_large_topk_edge_rows(gpu_ctx, oracle_mod, mode):
    """Constant rows (every element ties at the boundary), ascending and descending rows,
    -inf masks, and a row whose top-p cut lands exactly on a partial sum while the sums
    are inexact (the faithful check cannot prove the slot-order sum harmless there and
    re-runs the min-buffer)."""
    V, K = 6000, 2000
    cases = [("constant", np.zeros((3, V), np.float32)),
             ("ascending", (np.arange(V, dtype=np.float32) * 1e-3)[None, :].repeat(2, 0)),
             ("descending", (np.arange(V, dtype=np.float32)[::-1] * 1e-3)[None, :].repeat(2, 0).copy())]
    m = np.full((2, V), -np.inf, np.float32)
    m[:, ::7] = np.linspace(-3, 3, len(range(0, V, 7)), dtype=np.float32)
    cases.append(("neg_inf_mask", m))
    p = np.full((2, V), -60.0, np.float32)
    p[:, 1000:2000] = 0.0      # 1000 probabilities of exactly 1
    p[:, :1000] = -40.0        # 1000 tiny probabilities before them in index order
    cases.append(("planted_cut", p))
    for name, x in cases:
        B = x.shape[0]
        u = np.linspace(0.05, 0.95, B).astype(np.float32)
        for cfg in [default_config(temperature=1.0, top_k=K, top_p=0.5),
                    default_config(temperature=1.0, top_k=K),
                    default_config(temperature=0.7, top_k=V - 1, top_p=0.9)]:
            _check(gpu_ctx, oracle_mod, cfg, _t(x), u, mode=mode, label=f"{name} {cfg.as_dict()}")


def test_large_topk_host_entry(gpu_ctx, oracle_mod):
    """The same path through the host-buffer entry point."""
    rng = np.random.default_rng(5)
    B, V, K = 2, 100000, 4096
    x = (rng.normal(size=(B, V)) * 2).astype(np.float32)
    u = rng.random(B).astype(np.float32)
    cfg = default_config(temperature=1.0, top_k=K, top_p=0.95)
    gpu_ctx.set_tie_mode(abi.TIES_FAITHFUL)
    host = gpu_ctx.sample_host(cfg, x, u)
    o = oracle_run(oracle_mod, cfg, x, u, mode=abi.TIES_FAITHFUL)
    assert (host == o[0]).all()


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_large_topk_stage1_lists(gpu_ctx, oracle_mod, mode, dtype):
    """32 K <= V: the stream kernel's row lists feed the large top-k kernel. Batches of
    24 rows (several warps per row, lists that hold every element taken while the bounds
    rose) with smooth rows, rows of many ties at the bound (long lists), and a row whose
    list overflows (every element ties: the kernel re-selects from the whole row)."""
    import torch
    V, B = 262144, 24
    rng = np.random.default_rng(77 + (1 if dtype == "bf16" else 0))
    x = (rng.normal(size=(B, V)) * 2.0).astype(np.float32)
    x[B // 3: 2 * B // 3] = np.round(x[B // 3: 2 * B // 3] * 2) / 2
    x[-1] = 0.5
    xt = _t(x)
    if dtype == "bf16":
        xt = xt.to(torch.bfloat16)
    hist = rng.integers(0, V, size=(B, 64)).astype(np.int32)
    cnt = rng.integers(0, 65, size=B).astype(np.int32)
    u = rng.random(B).astype(np.float32)
    for cfg in [default_config(temperature=1.0, top_k=2000, top_p=0.9, repeat_penalty=1.2),
                default_config(temperature=0.8, top_k=4096, top_p=1.0, min_p=0.01),
                default_config(temperature=1.3, top_k=8192, top_p=0.95)]:
        _check(gpu_ctx, oracle_mod, cfg, xt, u, hist, cnt, mode, label=f"lists {dtype} {cfg.as_dict()}")
