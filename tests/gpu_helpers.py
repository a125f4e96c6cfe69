"""Helpers for the GPU parity tests: run the same seeded inputs through the CUDA library
(C ABI via vindexllm_b200.sampler) and through the CPU oracle."""
import os

import numpy as np

from vindexllm_b200 import abi

NTHREADS = max(1, min(32, os.cpu_count() or 1))


def to_host_bits(t):
    """torch CUDA tensor -> numpy float32 or uint16 (bf16 bits) with the same bits."""
    import torch
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).cpu().numpy().view(np.uint16)
    return t.float().cpu().numpy()


def gpu_run(ctx, cfg, logits, uniforms, history=None, count=None, mode=abi.TIES_FAITHFUL, out_k=0, vocab=None):
    import torch
    ctx.set_tie_mode(mode)
    dev = logits.device
    u = torch.as_tensor(np.ascontiguousarray(uniforms, np.float32), device=dev)
    tok, fl, oi, op = ctx.sample(cfg, logits, u, history, count, vocab=vocab, out_k=out_k, want_flags=True)
    torch.cuda.synchronize()
    res = [tok.cpu().numpy(), fl.cpu().numpy().view(np.uint32)]
    res.append(oi.cpu().numpy() if oi is not None else None)
    res.append(op.cpu().numpy() if op is not None else None)
    return res


def oracle_run(oracle_mod, cfg, logits, uniforms, history=None, count=None, mode=abi.TIES_FAITHFUL, out_k=0,
               vocab=None):
    x = to_host_bits(logits) if not isinstance(logits, np.ndarray) else logits
    h = None if history is None else (history.cpu().numpy() if not isinstance(history, np.ndarray) else history)
    c = None if count is None else (count.cpu().numpy() if not isinstance(count, np.ndarray) else count)
    return oracle_mod.sample_batch(cfg, np.ascontiguousarray(x), np.asarray(uniforms, np.float32), h, c, mode,
                                   out_k=out_k, nthreads=NTHREADS, vocab=vocab)


def flag_names(f):
    return [n for b, n in abi.FLAG_NAMES.items() if int(f) & b]


def compare(g, o, mode, strict_survivors=True, ignore_flags=0, label=""):
    """Asserts token and flag equality; survivors/probabilities in canonical mode."""
    gt, gf, gi, gp = g
    ot, of, oi, op = o
    gf = gf & ~np.uint32(abi.FLAG_FAITHFUL_PASS | ignore_flags)
    of = of & ~np.uint32(ignore_flags)
    bad = np.nonzero(gt != ot)[0]
    assert len(bad) == 0, f"{label}: {len(bad)} token mismatches, first rows {bad[:5]}: gpu {gt[bad[:5]]} " \
                          f"oracle {ot[bad[:5]]} flags {[flag_names(of[r]) for r in bad[:5]]}"
    badf = np.nonzero(gf != of)[0]
    assert len(badf) == 0, f"{label}: flag mismatch rows {badf[:5]}: gpu {[flag_names(gf[r]) for r in badf[:5]]} " \
                           f"oracle {[flag_names(of[r]) for r in badf[:5]]}"
    if gi is not None and mode == abi.TIES_CANONICAL and strict_survivors:
        assert (gi == oi).all(), f"{label}: survivor index mismatch"
        nz = op > 0
        rel = np.abs(gp[nz] - op[nz]) / op[nz]
        assert (gp[~nz] == 0).all() and (rel.max(initial=0) <= 1e-5), f"{label}: probability mismatch {rel.max()}"
