#!/usr/bin/env python
"""Benchmark of the token-sampling hot path (TVdxSampler.Process, src/VindexLLM.Sampler.pas).

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference] [--config c4]

One step = one sampling pass of the hot path over one batch of seeded synthetic logits
(the whole [B, V] batch, or each rank's vocab shard for N > 1). The default workload is
Benchmark configuration c4 (B=512, V=262144 fp32, T=1, top-k 64, top-p 0.95): the only
configuration defined for 1..8 GPUs, so every N runs the same total work (strong
scaling). At N=1 it is sampled unsharded; at N>1 each rank holds a contiguous vocab
shard, selects its local top-k, and the candidates are all-gathered with NCCL.

Rank 0 prints one JSON line. ``value`` is device-timed (inputs resident in HBM; the L2
is flushed between steps unless a step's input is at least twice the L2, and config.l2
says which; CUDA events around each step, max over ranks); ``e2e`` goes
through the host-buffer C-ABI call with the host->device copy of the logits and the
device->host copy of the tokens inside the timed region; ``cpu_baseline`` and
``--impl reference`` time the C++ restatement of TVdxSampler on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sampled tokens/sec at V=262144 (batch 1–1024); logits GB/s as % of HBM peak"
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="c4", choices=["c0", "c1", "c2", "c3", "c4"])
    ap.add_argument("--tie-mode", choices=["faithful", "canonical"], default="faithful")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--profile", action="store_true", help="only warmup + timed steps (for ncu launch lists)")
    ap.add_argument("--batch", type=int, default=None, help="override the config's batch (profiling only)")
    ap.add_argument("--no-flush", action="store_true", help="skip the L2 flush between steps (profiling only)")
    ap.add_argument("--no-configs", action="store_true", help="skip the per-configuration block (N=1)")
    ap.add_argument("--config-steps", type=int, default=30, help="timed steps per configuration in the block")
    return ap.parse_args()


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def load_traffic(name, world):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d.get(f"{name}_n{world}") or d.get(name)
    except Exception:
        return None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML, only while a timed region is
    open (``with sampler.region():``), so idle gaps between regions do not count."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, index, period=0.002, enabled=True):
        self.index, self.period = index, period
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._open = threading.Event()
        self._t = None
        self.ok = False
        if not enabled:
            return
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _sample(self):
        try:
            self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            for name, bit in self.REASONS.items():
                if r & bit:
                    self.reasons.add(name)
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            if self._open.wait(timeout=0.05):
                self._sample()
                time.sleep(self.period)

    def start(self):
        if self.ok and self._t is None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def stop(self):
        self._stop.set()
        self._open.set()
        if self._t:
            self._t.join()

    class _Region:
        def __init__(self, s):
            self.s = s

        def __enter__(self):
            if self.s.ok:
                self.s._open.set()
                self.s._sample()  # at least one sample per region
            return self

        def __exit__(self, *a):
            if self.s.ok:
                self.s._sample()
                self.s._open.clear()

    def region(self):
        return self._Region(self)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


L2_BYTES = 126 << 20  # B200 L2


def l2_policy(step_bytes):
    """(flush between steps?, description): a step that reads at least twice the L2
    needs no flush (what one step leaves in L2 is long evicted when the next step reaches
    it); a smaller one gets a 256 MiB write between steps, outside the step events."""
    if step_bytes >= 2 * L2_BYTES:
        return False, (f"no flush: each step reads {step_bytes / 2**20:.0f} MiB of logits, "
                       f"{step_bytes / L2_BYTES:.1f}x the 126 MiB L2")
    return True, "flushed between steps (256 MiB write, outside the per-step CUDA events)"


def workload_config(name, world, spec, tie_mode, l2_desc):
    cfg = {"workload": f"{name}: batch={spec['batch']} vocab=262144 {spec['dtype']} T={spec['temperature']} "
                       f"top_k={spec['top_k']} top_p={spec['top_p']} penalty={spec['repeat_penalty']} "
                       f"window={spec['window']} ({'vocab-sharded over %d GPUs' % world if world > 1 else 'unsharded'})",
           "batch": spec["batch"], "vocab": 262144, "logits_dtype": spec["dtype"], "top_k": spec["top_k"],
           "top_p": spec["top_p"], "temperature": spec["temperature"],
           "parallelism": f"vocab-shard{world}" if world > 1 else "single",
           "tie_mode": "canonical" if world > 1 else tie_mode,
           "l2": l2_desc}
    return cfg


def dominant_kernel(cfg, vocab, esz, batch):
    """Name of the library kernel that streams the logits for this configuration."""
    t = "float" if esz == 4 else "bf16"
    if batch <= 8 and (cfg.temperature == 0.0 or 0 < cfg.top_k < vocab):
        return f"vdxs::row_cluster_kernel<{t}> (one 8-CTA cluster per row, batch<=8)"
    if cfg.temperature == 0.0 or 0 < cfg.top_k < vocab:
        return f"vdxs::topk_stream_kernel<{t}> (stage-1 stream top-k)"
    return f"vdxs::full_max_kernel<{t}> + vdxs::full_sum_kernel<{t}> (full softmax)"


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ----------------------------------------------------------------------------------------
def preroll(torch, us):
    """A bounded spin on the device (torch.cuda._sleep counts clock cycles) queued ahead of
    a timed loop, so the host enqueues the loop while the device is busy: host launch
    latency and host scheduling jitter stay out of the device-timed steps."""
    torch.cuda._sleep(int(us * 2000))  # ~2 GHz SM clock: cycles for `us` microseconds


def timed_loop(torch, ctx, step, steps, flush, stream, clocks, staged_every=4, pre_us=None, align=None):
    """Runs `steps` timed steps with CUDA events around each on `stream`; the library
    records the stage events around its dominant pass on every `staged_every`-th step.
    Returns (per-step ms, mean dominant-kernel ms, launches)."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    staged = [j for j in range(steps) if j % staged_every == 0]
    kb = {j: torch.cuda.Event(enable_timing=True) for j in staged}
    ke = {j: torch.cuda.Event(enable_timing=True) for j in staged}
    for ev in list(kb.values()) + list(ke.values()):
        ev.record(stream)
    torch.cuda.synchronize()
    launches0 = ctx.launch_count()
    with clocks.region():
        preroll(torch, pre_us if pre_us is not None else min(200000, 60 * steps + 2000))
        if align is not None:
            align()  # a device-side collective after the pre-roll lines the ranks' timelines up
        for j in range(steps):
            if j in kb:
                ctx.set_stage_events(kb[j], ke[j])
            elif j % staged_every == 1:
                ctx.set_stage_events(None, None)
            starts[j].record(stream)
            step(j)
            ends[j].record(stream)
            if flush is not None:
                flush.zero_()
        torch.cuda.synchronize()
    ctx.set_stage_events(None, None)
    launches = ctx.launch_count() - launches0
    per_step = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    kern = statistics.mean(kb[j].elapsed_time(ke[j]) for j in staged)
    return per_step, kern, launches


def lat_summary(per_step_ms):
    lat = sorted(per_step_ms)
    p99 = lat[min(len(lat) - 1, int(round(0.99 * (len(lat) - 1))))]
    return {"mean": round(statistics.mean(lat) * 1e3, 2), "median": round(statistics.median(lat) * 1e3, 2),
            "p99": round(p99 * 1e3, 2)}


def host_bits(torch, x):
    import numpy as np
    return x.view(torch.int16).cpu().numpy().view(np.uint16) if x.dtype == torch.bfloat16 else x.cpu().numpy()


def oracle_parity(cfg, xh, u, hh, hc, mode, got, rows):
    """Tokens of `rows` (indices into the batch) against the CPU oracle in `mode`."""
    import numpy as np
    from oracle import oracle
    oracle.build()
    rows = np.asarray(rows)
    want, _, _, _ = oracle.sample_batch(cfg, np.ascontiguousarray(xh[rows]), np.ascontiguousarray(u[rows]),
                                        None if hh is None else np.ascontiguousarray(hh[rows]),
                                        None if hc is None else np.ascontiguousarray(hc[rows]), mode,
                                        nthreads=cpu_threads(), diag=False)
    bad = np.nonzero(np.asarray(got)[rows] != want)[0]
    return {"rows": int(len(rows)), "mismatches": int(len(bad)), "oracle_mode": "faithful" if mode == 0 else "canonical",
            "first_bad_rows": [int(rows[i]) for i in bad[:5]]}


def subset_rows(B, n=64):
    return list(range(B)) if B <= n else [int(i * B // n) for i in range(n)]


# Configurations timed in the same run as the headline line (N=1 only), each with its own
# oracle parity check: every target of the benchmark configurations in one JSON line.
CONFIG_BLOCK = [
    ("c0", "faithful", None),
    ("c1", "faithful", None),
    ("c2", "canonical", None),
    ("c2", "faithful", None),
    ("c2_greedy", "faithful", dict(top_k=1)),
    ("c3", "canonical", None),
    ("c3", "faithful", None),
]


def run_config_block(torch, ctx, dev, stream, clocks, peak, steps, warmup):
    import numpy as np
    from vindexllm_b200 import abi, synth
    out = {}
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for label, mode_name, over in CONFIG_BLOCK:
        name = label.split("_")[0]
        spec = synth.CONFIGS[name]
        cfg = synth.sampler_config(name, **(over or {}))
        mode = abi.TIES_FAITHFUL if mode_name == "faithful" else abi.TIES_CANONICAL
        ctx.set_tie_mode(mode)
        B, V = spec["batch"], synth.VOCAB
        if name == "c0":
            # 1000 steps, each with freshly seeded logits (1 GiB in all, above L2: no flush).
            S, W = 1000, 10
            xs = torch.empty((S + W, V), dtype=torch.float32, device=dev)
            for i in range(S + W):
                xs[i:i + 1].copy_(synth.make_logits("c0", step=i, device=str(dev)))
            u_all = torch.as_tensor(synth.make_uniforms("c0", S + W, batch=1), device=dev)
            tok = torch.empty((S + W, 1), dtype=torch.int32, device=dev)

            def step(i, xs=xs, u_all=u_all, tok=tok, cfg=cfg):
                ctx.sample(cfg, xs[i:i + 1], u_all[i], tokens=tok[i])
            for i in range(W):
                step(i)
            torch.cuda.synchronize()
            # The stage events (two extra records around the kernel) go on every 25th step:
            # at ~19 us per step they would otherwise weigh on the mean they help explain.
            per, kern, launches = timed_loop(torch, ctx, lambda j: step(W + j), S, None, stream, clocks,
                                             staged_every=25)
            got = tok[W:, 0].cpu().numpy()
            xh = host_bits(torch, xs[W:])
            par = oracle_parity(cfg, xh, u_all[W:, 0].cpu().numpy(), None, None, mode, got, list(range(S)))
            faithful_rows = None
            del xs
            esz, nsteps, l2 = 4, S, "1000 distinct freshly seeded rows (1 GiB, above L2), no flush"
        else:
            x = synth.make_logits(name, step=0, device=str(dev))
            h, c = synth.make_history(name, step=0, device=str(dev))
            S = steps
            u_all = torch.as_tensor(synth.make_uniforms(name, S + warmup + 1, batch=B), device=dev)
            tok = torch.empty(B, dtype=torch.int32, device=dev)

            def step(i, x=x, h=h, c=c, u_all=u_all, tok=tok, cfg=cfg):
                ctx.sample(cfg, x, u_all[i], h, c, tokens=tok)
            do_flush, l2 = l2_policy(x.numel() * x.element_size())
            fl_buf = flush if do_flush else None
            for i in range(warmup):
                step(i)
                if fl_buf is not None:
                    fl_buf.zero_()
            torch.cuda.synchronize()
            per, kern, launches = timed_loop(torch, ctx, lambda j: step(warmup + j), S, fl_buf, stream, clocks)
            # One more step outside the timed region, with flags: parity and emulated rows.
            tk, fl, _, _ = ctx.sample(cfg, x, u_all[S + warmup], h, c, want_flags=True)
            torch.cuda.synchronize()
            fl = fl.cpu().numpy().view(np.uint32)
            faithful_rows = int(((fl & abi.FLAG_FAITHFUL_PASS) != 0).sum())
            xh = host_bits(torch, x)
            par = oracle_parity(cfg, xh, u_all[S + warmup].cpu().numpy(), None if h is None else h.cpu().numpy(),
                                None if c is None else c.cpu().numpy(), mode, tk.cpu().numpy(), subset_rows(B))
            esz = x.element_size()
            nsteps = S
            del x
        ms = statistics.mean(per)
        alg = B * V * esz
        out[f"{label}_{mode_name}"] = {
            "batch": B, "dtype": "bf16" if esz == 2 else "f32", "top_k": cfg.top_k, "top_p": cfg.top_p,
            "temperature": cfg.temperature, "tie_mode": mode_name, "steps": nsteps, "l2": l2,
            "tokens_per_s": round(B / (ms / 1e3), 1), "ms_per_step": round(ms, 5), "latency_us": lat_summary(per),
            "dominant_kernel": {"name": dominant_kernel(cfg, V, esz, B), "ms": round(kern, 5),
                                "frac": round(alg / (kern / 1e3) / 1e9 / peak, 4), "alg_bytes": alg},
            "step_frac": round(alg / (ms / 1e3) / 1e9 / peak, 4),
            "gpu_launches_per_step": round(launches / nsteps, 2),
            "faithful_rows_per_step": faithful_rows, "parity": par}
        torch.cuda.empty_cache()
    return out


def run_unembed_block(torch, ctx, dev, stream, clocks, peak, steps=50):
    """The unembedding in front of the sampler (vdxs_sample_unembed_q4_0): a Gemma-3 sized
    tied embedding (262144 x 2560, Q4_0, 377 MB: above L2, no flush) times fresh hidden
    vectors each step, then c0's sampling configuration. The matvec alone is timed in a
    second loop for its fraction of the HBM peak (weight bytes per launch)."""
    import numpy as np
    from oracle import oracle
    from vindexllm_b200 import abi, synth
    from vindexllm_b200.sampler import Q4Weights
    V, H = synth.VOCAB, synth.HIDDEN
    wq = synth.make_q4_0(V, H, device=str(dev))
    w = Q4Weights(ctx, wq, H, V)
    wq_host = wq.cpu().numpy()
    del wq
    wbytes = V * (H // 32) * 18
    cfg = synth.sampler_config("c0")
    ctx.set_tie_mode(abi.TIES_FAITHFUL)
    out = {}
    for B in (1, 8):
        W = 5
        xs = torch.as_tensor(synth.make_hidden((steps + W + 1) * B, H), device=dev).view(steps + W + 1, B, H)
        us = torch.as_tensor(synth.make_uniforms("c0", steps + W + 1, batch=B), device=dev)
        tok = torch.empty(B, dtype=torch.int32, device=dev)
        logits = torch.empty(B, V, dtype=torch.float32, device=dev)
        for i in range(W):
            w.sample(cfg, xs[i], us[i], tokens=tok)
        torch.cuda.synchronize()
        per, _, launches = timed_loop(torch, ctx, lambda j: w.sample(cfg, xs[W + j], us[W + j], tokens=tok), steps,
                                      None, stream, clocks, staged_every=steps + 1)
        mv, _, _ = timed_loop(torch, ctx, lambda j: w.unembed(xs[W + j], logits), steps, None, stream, clocks,
                              staged_every=steps + 1)
        # One more step outside the timed regions, against the oracle (the shader's matvec,
        # then the restated sampler).
        xl = xs[steps + W]
        got = w.sample(cfg, xl, us[steps + W]).cpu().numpy()
        ol = oracle.matvec_q4_0(wq_host, xl.cpu().numpy(), nthreads=max(1, min(32, os.cpu_count() or 1)))
        ot = oracle.sample_batch(cfg, ol, us[steps + W].cpu().numpy(), None, None, abi.TIES_FAITHFUL,
                                 nthreads=B)[0]
        ms = statistics.mean(per)
        mv_ms = statistics.mean(mv)
        out[f"unembed_c0_b{B}"] = {
            "batch": B, "hidden": H, "vocab": V, "weights": "Q4_0 tied embedding, 377 MB (seeded)",
            "api": "vdxs_sample_unembed_q4_0", "steps": steps, "l2": "weights 3x the L2, no flush",
            "tokens_per_s": round(B / (ms / 1e3), 1), "ms_per_step": round(ms, 5), "latency_us": lat_summary(per),
            "dominant_kernel": {"name": "vdxs::q4_0_matvec_kernel (shader-order Q4_0 matvec)",
                                "ms": round(mv_ms, 5), "frac": round(wbytes / (mv_ms / 1e3) / 1e9 / peak, 4),
                                "alg_bytes": wbytes},
            "gpu_launches_per_step": round(launches / steps, 2),
            "parity": {"rows": B, "mismatches": int((got != ot).sum()), "oracle": "vdxo_matvec_q4_0 + vdxo_sample_batch"}}
        del xs
    w.close()
    return out


def run_ours(args, rank, world, local):
    import numpy as np
    import torch
    import torch.distributed as dist
    from vindexllm_b200 import abi, synth
    from vindexllm_b200.sampler import SamplerContext, ShardComm, broadcast_unique_id, shard_range

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    name = args.config
    spec = synth.CONFIGS[name]
    if world > 1 and name not in ("c4", "c1", "c2"):
        raise SystemExit("sharded benchmark runs c4 (or c1/c2)")
    if args.batch:
        spec = dict(spec, batch=args.batch)
    B, V = spec["batch"], synth.VOCAB
    cfg = synth.sampler_config(name)
    mode = abi.TIES_FAITHFUL if args.tie_mode == "faithful" else abi.TIES_CANONICAL
    mode = mode if world == 1 else abi.TIES_CANONICAL
    ctx = SamplerContext(local, tie_mode=mode)
    off, hi = shard_range(V, world, rank)
    x_full = synth.make_logits(name, step=0, batch=B, device=str(dev))
    check_rows = subset_rows(B)
    x_check = host_bits(torch, x_full[check_rows]) if rank == 0 and not args.profile else None
    x = x_full[:, off:hi].contiguous() if world > 1 else x_full
    if world > 1:
        del x_full
    esz = x.element_size()
    hist, hcnt = synth.make_history(name, step=0, batch=B, device=str(dev))
    nsteps = args.warmup + args.steps
    u_all = torch.as_tensor(synth.make_uniforms(name, nsteps + 1, batch=B), device=dev)
    tok = torch.empty(B, dtype=torch.int32, device=dev)
    comm = None
    if world > 1:
        comm = ShardComm(ctx, world, rank, broadcast_unique_id(rank))

    def step(i, tokens=tok):
        if comm is not None:
            comm.sample(cfg, x, off, V, u_all[i], hist, hcnt, tokens=tokens)
        else:
            ctx.sample(cfg, x, u_all[i], hist, hcnt, tokens=tokens)

    do_flush, l2_desc = l2_policy(x.numel() * esz)
    if args.no_flush:
        do_flush, l2_desc = False, "no flush (--no-flush: profiling only)"
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if do_flush else None
    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        step(i)
        if flush is not None:
            flush.zero_()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    # Clocks are sampled on rank 0 only: a polling thread on every rank adds host jitter.
    clocks = ClockSampler(local, enabled=(rank == 0)).start()
    align = None
    if world > 1:
        one = torch.ones(1, device=dev)
        align = lambda: dist.all_reduce(one)  # noqa: E731
    # A sharded step takes the host longer to enqueue (NCCL's non-blocking enqueue and
    # four launches) than the device needs to run it: the pre-roll must cover the
    # enqueue of every timed step, or later steps measure the host instead.
    pre_us = min(200000, (400 if world > 1 else 60) * args.steps + 2000)
    per_step, kern_ms, launches = timed_loop(torch, ctx, lambda j: step(args.warmup + j), args.steps, flush, stream,
                                             clocks, pre_us=pre_us, align=align)
    ctx.device_status()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    per = torch.tensor(per_step, dtype=torch.float64, device=dev)
    if world > 1:
        gathered = [torch.empty_like(per) for _ in range(world)]
        dist.all_gather(gathered, per)
        all_ranks = torch.stack(gathered).cpu().numpy()  # [world, steps]
    else:
        all_ranks = per.cpu().numpy()[None, :]
    total_ms = float(all_ranks.sum(axis=1).max())  # max over ranks of the timed region
    ms_per_step = total_ms / args.steps
    value = B / (ms_per_step / 1e3)
    step_max = all_ranks.max(axis=0)  # the slowest rank per step
    tail = []
    for r in range(all_ranks.shape[0]):
        med = float(np.median(all_ranks[r]))
        for j in np.nonzero(all_ranks[r] > 4 * med)[0]:
            tail.append({"rank": int(r), "step": int(j), "us": round(float(all_ranks[r, j]) * 1e3, 1),
                         "rank_median_us": round(med * 1e3, 1)})
    kt = torch.tensor([kern_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(kt, op=dist.ReduceOp.MAX)
    kern_ms = kt.item()

    # Parity of the timed configuration: one more step outside the timed region, a fixed
    # subset of rows against the CPU oracle (canonical ties when vocab-sharded).
    parity = None
    if not args.profile:
        step(nsteps)
        torch.cuda.synchronize()
        if rank == 0:
            hh = None if hist is None else hist.cpu().numpy()[check_rows]
            hc = None if hcnt is None else hcnt.cpu().numpy()[check_rows]
            got = tok.cpu().numpy()[check_rows]
            parity = oracle_parity(cfg, x_check, u_all[nsteps].cpu().numpy()[check_rows], hh, hc, mode, got,
                                   list(range(len(check_rows))))
            parity["rows_checked"] = f"{len(check_rows)} of {B} (every {max(1, B // len(check_rows))}th row)"

    # End to end through the public API with host buffers.
    e2e = None
    if not args.no_e2e and not args.profile:
        E = max(1, min(args.e2e_steps, args.steps))
        hx = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        hx.copy_(x)
        hu = torch.empty((E, B), dtype=torch.float32, pin_memory=True)
        hu.copy_(u_all[:E])
        hh = hist.cpu().pin_memory() if hist is not None else None
        hc = hcnt.cpu().pin_memory() if hcnt is not None else None
        if world == 1:
            hxn = hx.view(torch.int16).numpy().view("uint16") if x.dtype == torch.bfloat16 else hx.numpy()
            out = torch.empty(B, dtype=torch.int32, pin_memory=True).numpy()
            ctx.sample_host(cfg, hxn, hu[0].numpy(), None if hh is None else hh.numpy(),
                            None if hc is None else hc.numpy(), out=out)
            t0 = time.perf_counter()
            for j in range(E):
                ctx.sample_host(cfg, hxn, hu[j].numpy(), None if hh is None else hh.numpy(),
                                None if hc is None else hc.numpy(), out=out)
            el = time.perf_counter() - t0
        else:
            dx = torch.empty_like(x)
            du = torch.empty(B, dtype=torch.float32, device=dev)
            htok = torch.empty(B, dtype=torch.int32, pin_memory=True)
            dist.barrier()
            t0 = time.perf_counter()
            for j in range(E):
                dx.copy_(hx, non_blocking=True)
                du.copy_(hu[j], non_blocking=True)
                comm.sample(cfg, dx, off, V, du, hist, hcnt, tokens=tok)
                htok.copy_(tok, non_blocking=True)
                torch.cuda.current_stream().synchronize()
            el = time.perf_counter() - t0
        elt = torch.tensor([el], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(elt, op=dist.ReduceOp.MAX)
        el = elt.item()
        h2d = x.numel() * esz + B * 4
        e2e = {"value": round(B * E / el, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": B * 4, "steps": E,
               "api": "vdxs_sample_host" if world == 1 else "vdxs_sample_sharded + host copies",
               "bound": "PCIe host->device copy of the fp32 logits (h2d_bytes_per_step per step)"}

    # Product data flow (logits already on the device, as after the unembedding): the
    # stateful TVdxSampler mirror draws each row's uniform from its own xoshiro256**
    # stream, uploads them, samples and returns host tokens (vdxs_sampler_process).
    e2e_resident = None
    if world == 1 and not args.no_e2e and not args.profile:
        from vindexllm_b200.sampler import TVdxSampler
        ts = TVdxSampler(ctx, B)
        ts.SetConfig(synth.sampler_config(name, seed=7))
        if hist is not None:
            hh_np = hist.cpu().numpy()
            for j in range(hh_np.shape[1]):
                ts.AddToHistoryBatch(hh_np[:, j])
        E = max(1, min(args.e2e_steps * 10, args.steps))
        ts.Process(x)
        t0 = time.perf_counter()
        for _ in range(E):
            ts.Process(x)
        el = time.perf_counter() - t0
        ts.close()
        e2e_resident = {"value": round(B * E / el, 1), "unit": "tokens/s", "h2d_bytes_per_step": B * 4,
                        "d2h_bytes_per_step": B * 4, "steps": E,
                        "api": "TVdxSampler.Process on device-resident logits (vdxs_sampler_process)"}

    # Device-resident decode loop (vdxs_decode_step): row uniforms from device PRNG states,
    # sampling, history push and stop check, with no host round trip per token; one
    # synchronisation after the loop.
    device_decode = None
    if world == 1 and not args.no_e2e and not args.profile:
        from vindexllm_b200.sampler import DeviceDecodeState
        dcfg = synth.sampler_config(name, seed=7)
        W = dcfg.repeat_window
        dds = DeviceDecodeState(B, W, device=local, prng_states=[[7 + r, 11, 13, 17] for r in range(B)])
        if hist is not None and W > 0:
            n = min(W, hist.shape[1])
            dds.hist[:, :n].copy_(hist[:, :n])
            dds.count.fill_(n)
            dds.pos.fill_(n % W)
        E = max(1, min(args.e2e_steps * 10, args.steps))
        tok2 = torch.empty(B, dtype=torch.int32, device=dev)
        dds.step(ctx, dcfg, x, tokens=tok2)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(E):
            dds.step(ctx, dcfg, x, tokens=tok2)
        torch.cuda.synchronize()
        el = time.perf_counter() - t0
        device_decode = {"value": round(B * E / el, 1), "unit": "tokens/s", "steps": E,
                         "api": "vdxs_decode_step (PRNG, history ring and stop check on the device, "
                                "one synchronisation after the loop)"}
        # The same step captured once in a CUDA graph and replayed: no per-step launch work
        # on the host. One eager step of this state first, so the workspace no longer grows.
        gds = DeviceDecodeState(B, W, device=local, prng_states=[[7 + r, 11, 13, 17] for r in range(B)])
        gds.step(ctx, dcfg, x, tokens=tok2)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            gds.step(ctx, dcfg, x, tokens=tok2)
        graph.replay()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(E):
            graph.replay()
        torch.cuda.synchronize()
        el = time.perf_counter() - t0
        del graph
        device_decode["graph_replay"] = {"value": round(B * E / el, 1), "unit": "tokens/s",
                                         "us_per_step": round(el / E * 1e6, 2)}

    peak, peak_kind = load_peaks()
    # The dominant kernel reads every logit once; its other traffic (candidates out) is
    # below 1% of that and is not counted as algorithmic.
    alg_bytes = x.numel() * esz
    achieved = alg_bytes / (kern_ms / 1e3) / 1e9
    tr = load_traffic(name, world)
    if tr is None and world > 1:
        t1 = load_traffic(name, 1)
        if t1:
            # Stage-1 traffic is proportional to the elements read: scale to this shard.
            tr = {"bytes_per_launch": int(t1["bytes_per_launch"] * (hi - off) / V),
                  "source": t1["source"] + f"; scaled to this rank's shard ({hi - off} of {V})"}
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
            if peak_kind == "measured" else peak_kind,
            "traffic": tr.get("bytes_per_launch") if tr else None,
            "traffic_source": tr.get("source") if tr else None,
            "kernel": dominant_kernel(cfg, hi - off, esz, B),
            "kernel_ms": round(kern_ms, 5), "alg_bytes_per_launch": alg_bytes,
            "step_frac": round(B * V * esz / (ms_per_step / 1e3) / 1e9 / peak, 4)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.profile:
        cpu = cpu_baseline(name, cfg, x, hist, hcnt, u_all[0].cpu().numpy(), args.cpu_seconds)

    configs = None
    if world == 1 and not args.profile and not args.no_configs:
        configs = run_config_block(torch, ctx, dev, stream, clocks, peak, args.config_steps, 3)
        configs.update(run_unembed_block(torch, ctx, dev, stream, clocks, peak))
        ctx.set_tie_mode(mode)
    clocks.stop()

    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": spec["dtype"],
                "data": "synthetic (seeded; distribution of the named benchmark configuration)",
                "config": workload_config(name, world, spec, args.tie_mode, l2_desc),
                "latency_us": dict(lat_summary(step_max.tolist()), mean=round(ms_per_step * 1e3, 2)),
                "latency_note": "per step: the slowest rank's CUDA-event time; mean = max over ranks of the "
                                "summed timed region / steps" if world > 1 else "per step: CUDA-event time",
                "tail_steps_over_4x_median": tail,
                "logits_gbs": round(B * V * esz / (ms_per_step / 1e3) / 1e9, 1),
                "gpu_launches": launches,
                "parity": parity,
                "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "e2e_resident_logits": e2e_resident,
                "device_decode": device_decode,
                "configs": configs,
                "clocks": clocks.summary()}
        print(json.dumps(line), flush=True)
    if comm is not None:
        comm.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


def cpu_baseline(name, cfg, x, hist, hcnt, u, seconds):
    """C++ restatement of TVdxSampler (the oracle, faithful mode) on the host cores."""
    import numpy as np
    import torch
    from oracle import oracle
    from vindexllm_b200 import abi
    oracle.build()
    xh = x.view(torch.int16).cpu().numpy().view(np.uint16) if x.dtype == torch.bfloat16 else x.cpu().numpy()
    hh = None if hist is None else hist.cpu().numpy()
    hc = None if hcnt is None else hcnt.cpu().numpy()
    nt = cpu_threads()
    rows_done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        oracle.sample_batch(cfg, xh, u, hh, hc, abi.TIES_FAITHFUL, nthreads=nt, diag=False)
        rows_done += xh.shape[0]
    el = time.perf_counter() - t0
    return {"value": round(rows_done / el, 1), "unit": "tokens/s", "cores": nt, "kind": "port",
            "sample": f"{rows_done} rows of {name} step 0 ({xh.shape[0]} rows per call) over {el:.1f} s, "
                      f"C++ restatement of TVdxSampler.Process, rows split across {nt} threads"}


# ----------------------------------------------------------------------------------------
def run_reference(args, rank, world):
    """The reference's CPU implementation of the path (C++ restatement of TVdxSampler:
    the Delphi original cannot be compiled here) on all host threads, rank 0 only."""
    if rank != 0:
        return
    import numpy as np
    from oracle import oracle
    from vindexllm_b200 import abi, synth
    oracle.build()
    name = args.config
    spec = synth.CONFIGS[name]
    cfg = synth.sampler_config(name)
    B, V = spec["batch"], synth.VOCAB
    x = synth.make_logits(name, step=0, device="cpu")
    import torch
    xh = x.view(torch.int16).numpy().view(np.uint16) if x.dtype == torch.bfloat16 else x.numpy()
    hist, hcnt = synth.make_history(name, step=0, device="cpu")
    hh = None if hist is None else hist.numpy()
    hc = None if hcnt is None else hcnt.numpy()
    u = synth.make_uniforms(name, args.warmup + args.steps, batch=B)
    nt = cpu_threads()
    # Bound each step so the whole run stays within a few minutes.
    t0 = time.perf_counter()
    oracle.sample_batch(cfg, xh, u[0], hh, hc, abi.TIES_FAITHFUL, nthreads=nt, diag=False)
    est = time.perf_counter() - t0
    budget = 120.0 / max(1, args.steps + args.warmup)
    rows = B if est <= budget else max(nt, int(B * budget / est) // nt * nt)
    rows = min(rows, B)
    xs = np.ascontiguousarray(xh[:rows])
    hs = None if hh is None else np.ascontiguousarray(hh[:rows])
    cs = None if hc is None else np.ascontiguousarray(hc[:rows])
    for i in range(args.warmup):
        oracle.sample_batch(cfg, xs, u[i][:rows], hs, cs, abi.TIES_FAITHFUL, nthreads=nt, diag=False)
    t0 = time.perf_counter()
    for j in range(args.steps):
        oracle.sample_batch(cfg, xs, u[args.warmup + j][:rows], hs, cs, abi.TIES_FAITHFUL, nthreads=nt, diag=False)
    el = time.perf_counter() - t0
    ms = el * 1e3 / args.steps
    value = rows / (ms / 1e3)
    sample = (f"{rows} of {B} rows of {name} per step, C++ restatement of TVdxSampler.Process "
              f"(Delphi original not compilable here), rows split across {nt} threads")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": spec["dtype"],
            "data": "synthetic (seeded; distribution of the named benchmark configuration)",
            "config": workload_config(name, world, spec, "faithful",
                                      l2_policy(B * (V // world) * (2 if spec["dtype"] == "bf16" else 4))[1]),
            "cpu_baseline": {"value": round(value, 1), "unit": "tokens/s", "cores": nt, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and "RANK" in os.environ:
        args.gpus = world
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1 and "RANK" not in os.environ:
        raise SystemExit("for --gpus N > 1 launch with torch.distributed.run (one process per GPU)")
    run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
