#!/usr/bin/env python
"""Benchmark of the token-sampling hot path (TVdxSampler.Process, src/VindexLLM.Sampler.pas).

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference] [--config c4]

One step = one sampling pass of the hot path over one batch of seeded synthetic logits
(the whole [B, V] batch, or each rank's vocab shard for N > 1). The default workload is
BASELINE config c4 (B=512, V=262144 fp32, T=1, top-k 64, top-p 0.95): the only
configuration defined for 1..8 GPUs, so every N runs the same total work (strong
scaling). At N=1 it is sampled unsharded; at N>1 each rank holds a contiguous vocab
shard, selects its local top-k, and the candidates are all-gathered with NCCL.

Rank 0 prints one JSON line. ``value`` is device-timed (inputs resident in HBM, L2
flushed between steps, CUDA events around each step, max over ranks); ``e2e`` goes
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
    """Samples SM clock and clock-event reasons through NVML while the timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, index, period=0.005):
        self.index, self.period = index, period
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._t = None
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def workload_config(name, world, spec, tie_mode):
    cfg = {"workload": f"{name}: batch={spec['batch']} vocab=262144 {spec['dtype']} T={spec['temperature']} "
                       f"top_k={spec['top_k']} top_p={spec['top_p']} penalty={spec['repeat_penalty']} "
                       f"window={spec['window']} ({'vocab-sharded over %d GPUs' % world if world > 1 else 'unsharded'})",
           "batch": spec["batch"], "vocab": 262144, "logits_dtype": spec["dtype"], "top_k": spec["top_k"],
           "top_p": spec["top_p"], "temperature": spec["temperature"],
           "parallelism": f"vocab-shard{world}" if world > 1 else "single",
           "tie_mode": "canonical" if world > 1 else tie_mode,
           "l2": "flushed between steps (256 MiB write, outside the per-step CUDA events)"}
    return cfg


def dominant_kernel(cfg, vocab, esz, batch):
    """Name of the library kernel that streams the logits for this configuration."""
    t = "float" if esz == 4 else "bf16"
    if batch <= 8 and (cfg.temperature == 0.0 or 0 < cfg.top_k < vocab):
        return f"vdxs::row_cluster_kernel<{t}> (one 8-CTA cluster per row, batch<=8)"
    if cfg.temperature == 0.0 or 0 < cfg.top_k <= 128:
        return f"vdxs::topk_hist_kernel<{t}> (stage-1 stream top-k, k<=128)"
    if 0 < cfg.top_k < vocab:
        return f"vdxs::topk_wide_kernel<{t}> (stage-1 stream top-k, 128<k<=1024)"
    return f"vdxs::full_max_kernel<{t}> + vdxs::full_sum_kernel<{t}> (full softmax)"


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ----------------------------------------------------------------------------------------
def run_ours(args, rank, world, local):
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
    ctx = SamplerContext(local, tie_mode=mode if world == 1 else abi.TIES_CANONICAL)
    off, hi = shard_range(V, world, rank)
    x_full = synth.make_logits(name, step=0, batch=B, device=str(dev))
    x = x_full[:, off:hi].contiguous() if world > 1 else x_full
    if world > 1:
        del x_full
    esz = x.element_size()
    hist, hcnt = synth.make_history(name, step=0, batch=B, device=str(dev))
    nsteps = args.warmup + args.steps
    u_all = torch.as_tensor(synth.make_uniforms(name, nsteps, batch=B), device=dev)
    tok = torch.empty(B, dtype=torch.int32, device=dev)
    comm = None
    if world > 1:
        comm = ShardComm(ctx, world, rank, broadcast_unique_id(rank))

    def step(i):
        if comm is not None:
            comm.sample(cfg, x, off, V, u_all[i], hist, hcnt, tokens=tok)
        else:
            ctx.sample(cfg, x, u_all[i], hist, hcnt, tokens=tok)

    flush = torch.empty(16 if args.no_flush else 256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        step(i)
        flush.zero_()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    # The library records these around its dominant pass over the logits in each step.
    kb = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ke = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for ev in kb + ke:
        ev.record(stream)
    torch.cuda.synchronize()
    launches0 = ctx.launch_count()
    clocks = ClockSampler(local)
    # The stage events are recorded on every 4th timed step only: each pair adds two
    # event records to the step it brackets.
    staged = [j for j in range(args.steps) if j % 4 == 0]
    with clocks:
        for j in range(args.steps):
            if j % 4 == 0:
                ctx.set_stage_events(kb[j], ke[j])
            elif j % 4 == 1:
                ctx.set_stage_events(None, None)
            starts[j].record(stream)
            step(args.warmup + j)
            ends[j].record(stream)
            flush.zero_()
        torch.cuda.synchronize()
    ctx.set_stage_events(None, None)
    launches = ctx.launch_count() - launches0
    ctx.device_status()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    per_step = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = torch.tensor([sum(per_step)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(total_ms, op=dist.ReduceOp.MAX)
    ms_per_step = total_ms.item() / args.steps
    value = B / (ms_per_step / 1e3)
    lat = sorted(per_step)
    p99 = lat[min(len(lat) - 1, int(round(0.99 * (len(lat) - 1))))]
    kt = torch.tensor([statistics.mean(kb[j].elapsed_time(ke[j]) for j in staged)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(kt, op=dist.ReduceOp.MAX)
    kern_ms = kt.item()

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
        e2e = {"value": B * E / el, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": B * 4,
               "steps": E, "api": "vdxs_sample_host" if world == 1 else "vdxs_sample_sharded + host copies"}

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
        # on the host.
        gds = DeviceDecodeState(B, W, device=local, prng_states=[[7 + r, 11, 13, 17] for r in range(B)])
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
    # below 0.1% of that and is not counted as algorithmic.
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
            "kernel_ms": round(kern_ms, 5), "kernel_ms_steps": len(staged), "alg_bytes_per_launch": alg_bytes,
            "step_frac": round(B * V * esz / (ms_per_step / 1e3) / 1e9 / peak, 4)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.profile:
        cpu = cpu_baseline(name, cfg, x, hist, hcnt, u_all[0].cpu().numpy(), args.cpu_seconds)

    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": spec["dtype"],
                "data": "synthetic (seeded; distribution of the named BASELINE config)",
                "config": workload_config(name, world, spec, args.tie_mode),
                "latency_us_per_step": round(ms_per_step * 1e3, 2),
                "latency_us": {"mean": round(ms_per_step * 1e3, 2), "median": round(statistics.median(per_step) * 1e3, 2),
                               "p99": round(p99 * 1e3, 2)},
                "logits_gbs": round(B * V * esz / (ms_per_step / 1e3) / 1e9, 1),
                "gpu_launches": launches,
                "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "e2e_resident_logits": e2e_resident,
                "device_decode": device_decode,
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
            "data": "synthetic (seeded; distribution of the named BASELINE config)",
            "config": workload_config(name, world, spec, "faithful"),
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
