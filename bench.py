#!/usr/bin/env python
"""Benchmark of the paged-attention decode path; prints ONE JSON line.

    python bench.py [--gpus N --steps K --warmup W --workload NAME --impl b200|reference]

N > 1 runs under torch.distributed.run, one rank per GPU.  A step is one
decode call over one batch of the workload (default llama8b_gqa: 64 sequences
x 4096 tokens, 32/8 heads, D 128, bs 16, bf16 — 1 GiB of KV, larger than the
126 MB L2, so no flush is needed between steps).  At N > 1 the same batch is
split over the ranks ("strong" scaling, total work fixed): its sequences are
sharded by tokens with no collective on the data path (--mode shard, the
default), or, for long_context, every context is split into token ranges and
the ranks' partial states are merged over NVLink (--mode split).  --mode
replicate gives every rank a batch of its own instead ("weak" scaling).

value     KV-cache bytes read by all ranks / max-over-ranks device time of the K
          steps (CUDA events around the public wrapper, inputs resident).
roofline  algorithmic KV bytes per decode-kernel launch / the kernel's mean
          event-timed duration, against the measured HBM copy bandwidth.
e2e       the same metric through the public wrapper with the step's inputs
          (query, cache_seqlens, block_table) copied from pinned host memory
          and the output read back every step; the KV cache stays resident.
--impl reference  the reference's CPU path (src/kernel_eager.py in fp32) on the
          host cores, on a bounded sample per step: the faster of its torch
          restatement (oracle/eager_torch.py, the reference's own operations)
          and its numpy restatement (oracle/eager.py).
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "KV-cache read GB/s (% of B200 HBM peak) and µs per paged-decode call"
UNIT = "GB/s"
FALLBACK_HBM_GBS = 6650.0
DATASHEET_HBM_GBS = 8000.0  # B200 HBM3e nominal (DGX figure), for context


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", default="llama8b_gqa")
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="wall budget of the CPU-baseline sample (rank 0, N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=200)
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="split mode's state exchange: p2p = one fused kernel that stores the "
                         "states into peer memory and merges (CUDA IPC buffers); nccl = NCCL "
                         "all-gather, then the merge kernel")
    ap.add_argument("--mode", choices=["replicate", "shard", "split"], default=None,
                    help="N>1: shard = one batch's sequences split over ranks (strong "
                         "scaling); split = every sequence's context split over ranks, "
                         "states merged over NVLink (strong); replicate = every rank its own "
                         "batch (weak).  Default: split for long_context, else shard")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def hbm_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, STREAM-style copy)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback 6.65 TB/s (MEASURED_PEAKS.json absent)"


def ncu_traffic(workload):
    """DRAM bytes per decode-kernel launch from the committed ncu summary."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    try:
        d = json.loads(p.read_text())[workload]
        return d["dram_bytes_per_launch"], d.get("source")
    except Exception:
        return None, None


class ClockSampler:
    """Samples SM clock, power and clock-event reasons through NVML while the
    timed region runs (read-only; nothing is set)."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        "display_clock_setting": 0x100,
    }

    def __init__(self, torch_device, period_s=0.02):
        self.samples = []
        self.period = period_s
        self._stop = threading.Event()
        self.handle = None
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            import torch
            props = torch.cuda.get_device_properties(torch_device)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            try:
                self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(torch_device.index or 0)
            self.nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # NVML missing: report no clocks
            self.error = str(e)

    def _run(self):
        n = self.nvml
        while not self._stop.is_set():
            try:
                sm = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
                reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                power = n.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
                self.samples.append((time.time(), sm, reasons, power))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.handle is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.handle is not None:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        sms = [s[1] for s in self.samples]
        mask = 0
        for s in self.samples:
            mask |= s[2]
        reasons = [k for k, v in self.REASONS.items() if mask & v and k != "gpu_idle"]
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(sms),
                "power_w_max": round(max(s[3] for s in self.samples), 1)}


class CpuRestatements:
    """The reference's CPU decode (src/kernel_eager.py:29-56, fp32) on the
    first ``num_seqs`` sequences of a workload, in its two restatements:
    ``torch`` (oracle/eager_torch.py: the reference's own torch operations,
    one kv head at a time, torch's CPU threads) and ``numpy``
    (oracle/eager.py: a thread pool over heads, one BLAS thread each)."""

    def __init__(self, workload, seed, num_seqs, threads):
        import torch

        from pagedattention_b200.workloads import make_inputs
        torch.set_num_threads(threads)
        self.threads = threads
        inp = make_inputs(workload, seed=seed, num_seqs=num_seqs)
        q, k, v, sl, bt = inp.reference_layout()
        self.t = (q.float(), k.float(), v.float(), sl, bt.contiguous())
        self.n = tuple(x.numpy() for x in self.t)
        self.scale = inp.scale
        self.kv_bytes = inp.kv_bytes()
        self.num_seqs = num_seqs

    def run(self, kind):
        from oracle import eager, eager_torch
        if kind == "torch":
            eager_torch.flash_attn_with_kvcache(*self.t, self.scale)
        else:
            eager.flash_attn_with_kvcache(*self.n, self.scale, threads=self.threads)

    def seconds(self, kind, reps):
        self.run(kind)  # warm
        t0 = time.perf_counter()
        for _ in range(reps):
            self.run(kind)
        return (time.perf_counter() - t0) / reps

    def faster(self, reps=2):
        """(kind of the faster restatement, {kind: GB/s}) on this sample."""
        gbs = {k: self.kv_bytes / self.seconds(k, reps) / 1e9 for k in ("torch", "numpy")}
        return max(gbs, key=gbs.get), gbs


RESTATEMENT_NAMES = {"torch": "torch restatement of the reference's eager ops (oracle/eager_torch.py)",
                     "numpy": "numpy restatement, thread pool over heads (oracle/eager.py)"}


def host_cores():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def sample_seqs(workload, seed, seconds_per_call, threads):
    """Sequences of the workload whose CPU decode takes about
    ``seconds_per_call`` with the slower restatement (calibrated on one)."""
    one = CpuRestatements(workload, seed, 1, threads)
    per_seq = max(max(one.seconds(k, 1) for k in ("torch", "numpy")), 1e-4)
    return max(1, min(workload.num_seqs, int(seconds_per_call / per_seq)))


def cpu_oracle_sample(workload, seed, budget_s, threads):
    """Time the reference's CPU decode (fp32) on the first sequences of the
    workload, both restatements; the faster is the baseline.

    Returns (GB/s over algorithmic KV bytes, description, cores, {kind: GB/s})."""
    nseq = sample_seqs(workload, seed, budget_s / 8, threads)
    r = CpuRestatements(workload, seed, nseq, threads)
    best, gbs = r.faster(reps=3)
    desc = (f"first {nseq} of {workload.num_seqs} sequences of {workload.name} "
            f"({r.kv_bytes / 1e6:.1f} MB of KV), fp32; faster of two restatements of "
            f"src/kernel_eager.py: {RESTATEMENT_NAMES[best]}, 3 timed reps")
    return gbs[best], desc, threads, gbs


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return  # the CPU reference arm runs on rank 0 only
    from pagedattention_b200.workloads import WORKLOADS

    w = WORKLOADS[args.workload]
    cores = host_cores()
    # Size each step so warmup + steps finish in about two minutes.
    budget_per_step = max(0.02, 120.0 / (args.steps + args.warmup))
    nseq = sample_seqs(w, args.seed, budget_per_step, cores)
    r = CpuRestatements(w, args.seed, nseq, cores)
    best, gbs = r.faster(reps=1)
    for _ in range(args.warmup):
        r.run(best)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        r.run(best)
    dt = time.perf_counter() - t0
    value = r.kv_bytes * args.steps / dt / 1e9
    sample = (f"first {nseq} of {w.num_seqs} sequences of {w.name} per step "
              f"({r.kv_bytes / 1e6:.1f} MB of KV), fp32; the faster of two restatements of "
              f"src/kernel_eager.py on this sample: {RESTATEMENT_NAMES[best]}")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": w.name, "description": w.description, "sample_seqs": nseq,
                   "device": "cpu"},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample,
                         "restatements_gbs": {k: round(v, 3) for k, v in gbs.items()}},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    emit(line)


def run_b200(args):
    import torch
    import torch.distributed as dist

    from pagedattention_b200 import flash_attn_with_kvcache_wrapper_b200 as decode
    from pagedattention_b200 import paged_attention
    from pagedattention_b200.distributed import (PeerExchange, context_ranges,
                                                 decode_context_parallel, lens_of_units,
                                                 shard_heads, shard_sequences)
    from pagedattention_b200.kernel_b200 import kernel_events, launches_per_call
    from pagedattention_b200.workloads import WORKLOADS, make_inputs, sample_lens

    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x):
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    w = WORKLOADS[args.workload]
    mode = args.mode or ("split" if w.name == "long_context" else "shard")
    if world == 1:
        mode = "replicate"
    elt = 2
    lens_all = sample_lens(w, args.seed)
    global_bytes = int(lens_all.to(torch.int64).sum()) * w.num_kv_heads * w.head_size * elt * 2
    if mode == "replicate":      # every rank decodes its own batch
        inp = make_inputs(w, seed=args.seed + rank, device=dev, gen_device=dev)
        parallelism = f"dp{world} (independent sequence batches per rank, no collective)"
    elif mode == "shard" and len(lens_all) >= world:  # sequences split over ranks (LPT)
        idx = shard_sequences(lens_all.tolist(), world)[rank]
        inp = make_inputs(w, seed=args.seed + rank, device=dev, gen_device=dev,
                          lens=lens_all[idx])
        parallelism = f"sequence-sharded over {world} ranks (LPT by tokens), no collective"
    elif mode == "shard":        # fewer sequences than ranks: (sequence, kv head) units
        inp = make_inputs(w, seed=args.seed, device=dev, gen_device=dev, lens=lens_all)
        lens2d = lens_all[:, None].expand(len(lens_all), w.num_kv_heads)
        head_units = shard_heads(lens2d, world)[rank]
        parallelism = (f"(sequence, kv head)-sharded over {world} ranks (LPT by tokens), "
                       "no collective")
    else:                        # every context split over ranks, states merged over NCCL
        starts, ends = context_ranges(lens_all, world, w.partition_tokens or 512)
        inp = make_inputs(w, seed=args.seed, device=dev, gen_device=dev,
                          lens=(ends[rank] - starts[rank]).to(torch.int32))
        parallelism = (f"context split over {world} ranks ({w.partition_tokens or 512}-token "
                       "aligned ranges), " + (
                           "(o, lse) states stored into peer memory and merged by one fused "
                           "kernel" if args.exchange == "p2p" else
                           "(o, lse) states all-gathered over NCCL and merged"))
    q, k, v, sl, bt = inp.reference_layout()
    bt = bt.contiguous()
    kv_bytes = inp.kv_bytes()
    if mode == "shard" and len(lens_all) < world:
        sl = lens_of_units(sl.cpu(), head_units).to(torch.int32).to(dev)
        kv_bytes = int(sl.to(torch.int64).sum()) * w.head_size * elt * 2
    total_bytes = kv_bytes * world if mode == "replicate" else global_bytes
    L2 = torch.cuda.get_device_properties(dev).L2_cache_size
    # Keep every step's KV out of L2: workloads whose KV is under 3x L2
    # rotate over enough independent copies of the cache (same block table)
    # that the KV read by consecutive steps together exceeds 3x L2.
    pool_bytes = k.numel() * k.element_size() * 2
    copies = max(1, -(-3 * L2 // kv_bytes)) if kv_bytes <= 3 * L2 else 1
    caches = [(k, v)] + [(k.clone(), v.clone()) for _ in range(copies - 1)]
    if copies == 1:
        l2_note = (f"inputs larger than L2 ({kv_bytes / 2**20:.0f} MiB KV per step vs "
                   f"{L2 / 2**20:.0f} MiB L2), no flush")
    else:
        l2_note = (f"{kv_bytes / 2**20:.0f} MiB KV per step < 3x L2 ({L2 / 2**20:.0f} MiB): steps "
                   f"rotate over {copies} copies of the cache ({copies * kv_bytes / 2**20:.0f} MiB "
                   f"of KV read per rotation)")
    step_no = [0]
    exchange = None
    if mode == "split" and args.exchange == "p2p":
        exchange = PeerExchange(*q[:, 0].shape)

    kpool_copies = [(inp.k_pool, inp.v_pool)] + [
        (kc.view_as(inp.k_pool), vc.view_as(inp.v_pool)) for kc, vc in caches[1:]]

    def run(qx, slx, btx, seq_bt, seq_lens):
        i = step_no[0] % copies
        step_no[0] += 1
        if mode == "split":
            kp, vp = kpool_copies[i]
            return decode_context_parallel(qx[:, 0], kp, vp, seq_bt, seq_lens, inp.scale,
                                           w.block_size, exchange=exchange)
        kc, vc = caches[i]
        return decode(qx, kc, vc, slx, btx, inp.scale)

    seq_bt, seq_lens = inp.block_tables, inp.context_lens

    def step():
        return run(q, sl, bt, seq_bt, seq_lens)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()

    K = args.steps
    launches = launches_per_call(q, k, v, sl, bt, inp.scale)
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(dev)
    with sampler:
        t_start.record()
        for _ in range(K):
            step()
        t_end.record()
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    elapsed_ms = max_over_ranks(t_start.elapsed_time(t_end))
    ms_per_step = elapsed_ms / K
    value = total_bytes * K / (elapsed_ms / 1e3) / 1e9

    # Kernel-only timing for the roofline: the same K steps again, with the
    # library recording an event pair around every decode-kernel launch on
    # the launching stream.  (A separate pass, because recording events
    # between the planner and decode launches disables their overlap.)
    kb = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ka = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    for e in kb + ka:
        e.record()  # create the events before the timed pass
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    for i in range(K):
        with kernel_events(kb[i], ka[i]):
            step()
    torch.cuda.synchronize()
    barrier()
    kernel_ms = statistics.fmean(b.elapsed_time(a) for b, a in zip(kb, ka))
    # per-GPU kernel throughput of the slowest rank
    achieved = -max_over_ranks(-(kv_bytes / (kernel_ms / 1e3) / 1e9))
    kernel_ms = max_over_ranks(kernel_ms)

    # The same calls captured once in a CUDA graph and replayed: the device
    # time per call without any host work (one captured call per cache copy,
    # so the L2 rotation is kept).  One GPU only: no process group is active
    # while the stream is captured.
    graph_line = None
    if world == 1:
        gstream = torch.cuda.Stream(dev)
        gstream.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(gstream):
            step()
            gstream.synchronize()
            with torch.cuda.graph(graph, stream=gstream, capture_error_mode="thread_local"):
                for _ in range(copies):
                    step()
        torch.cuda.current_stream(dev).wait_stream(gstream)
        reps = max(1, -(-min(K, 200) // copies))
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(reps):
            graph.replay()
        g1.record()
        torch.cuda.synchronize()
        graph_ms = max_over_ranks(g0.elapsed_time(g1)) / (reps * copies)
        graph_line = {"us_per_call": round(graph_ms * 1e3, 2),
                      "value": round(total_bytes / (graph_ms / 1e3) / 1e9, 1), "unit": UNIT,
                      "calls": reps * copies,
                      "note": "the public wrapper's calls captured once in a CUDA graph and "
                              "replayed: device time per call with no host work"}
        del graph

    # e2e: every step copies its inputs from pinned host memory and reads its
    # output back, as a serving loop does: each step's inputs are staged on a
    # copy stream (two device buffers, so a copy overlaps the previous
    # step's decode), the step decodes into one of two preallocated outputs
    # through the in-place public call (paged_attention, or the context
    # split's decode_context_parallel with out=), and each output returns on
    # a third stream.  The KV cache stays resident.  (split mode: the
    # per-rank block table and lengths of its token range)
    if mode == "split":
        ins = [q, seq_lens, seq_bt]
    else:
        ins = [q, sl, bt]
    # The step's inputs share one pinned staging buffer (256-byte aligned
    # slots), so each step stages them with a single host-to-device copy into
    # one of two device buffers; the wrapper gets views of the device buffer.
    offs, total_in = [], 0
    for t in ins:
        offs.append(total_in)
        total_in += (t.numel() * t.element_size() + 255) // 256 * 256
    host_pack = torch.empty(total_in, dtype=torch.uint8).pin_memory()
    dev_packs = [torch.empty(total_in, dtype=torch.uint8, device=dev) for _ in range(2)]

    def views(buf):
        return [buf[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
                for o, t in zip(offs, ins)]

    hosts = views(host_pack)
    for h, t in zip(hosts, ins):
        h.copy_(t.cpu())
    devs = [views(b) for b in dev_packs]
    out_shape = q[:, 0].shape
    out_h = [torch.empty(out_shape, dtype=q.dtype).pin_memory() for _ in range(2)]
    out_d = [torch.empty(out_shape, dtype=q.dtype, device=dev) for _ in range(2)]
    compute = torch.cuda.current_stream(dev)
    h2d_stream, d2h_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    staged = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]
    for e in freed:
        e.record(compute)
    e2e_no = [0]

    def run_into(out, qx, slx, btx, seq_bt, seq_lens):
        i = step_no[0] % copies
        step_no[0] += 1
        if mode == "split":
            kp, vp = kpool_copies[i]
            decode_context_parallel(qx[:, 0], kp, vp, seq_bt, seq_lens, inp.scale,
                                    w.block_size, exchange=exchange, out=out)
        else:
            kc, vc = caches[i]
            paged_attention(out, qx[:, 0], kc, vc, btx, slx, inp.scale, w.block_size)

    def e2e_step():
        b = e2e_no[0] % 2
        e2e_no[0] += 1
        h2d_stream.wait_event(freed[b])
        with torch.cuda.stream(h2d_stream):
            dev_packs[b].copy_(host_pack, non_blocking=True)
        staged[b].record(h2d_stream)
        compute.wait_event(staged[b])
        if mode == "split":
            run_into(out_d[b], devs[b][0], None, None, devs[b][2], devs[b][1])
        else:
            run_into(out_d[b], devs[b][0], devs[b][1], devs[b][2], None, None)
        freed[b].record(compute)
        d2h_stream.wait_event(freed[b])
        with torch.cuda.stream(d2h_stream):
            out_h[b].copy_(out_d[b], non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    E = max(1, min(args.e2e_steps, K))
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(compute)
    for _ in range(E):
        e2e_step()
    compute.wait_stream(d2h_stream)
    e1.record(compute)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = total_bytes * E / (e2e_ms / 1e3) / 1e9
    h2d = total_in  # the packed copy, slot padding included
    d2h = out_h[0].numel() * out_h[0].element_size()

    exchange_status = None
    if exchange is not None:
        exchange_status = exchange.read_status()
        exchange.close()
        if exchange_status:
            raise SystemExit(f"rank {rank}: peer exchange status {exchange_status:#x}")
    # bytes moved besides the K/V pages (this rank's call): q read, output
    # written, block-table entries and lengths read
    extra_bytes = {"q": q.numel() * q.element_size(), "out": q.numel() * q.element_size(),
                   "block_table": int(((sl.to(torch.int64) + w.block_size - 1) // w.block_size).sum()) * 4,
                   "seqlens": sl.numel() * sl.element_size()}
    peak, peak_src = hbm_peak()
    traffic, traffic_src = ncu_traffic(w.name)
    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            gbs, desc, used, both = cpu_oracle_sample(w, args.seed, args.cpu_seconds,
                                                      host_cores())
            cpu = {"value": round(gbs, 3), "unit": UNIT, "cores": used, "kind": "port",
                   "sample": desc, "restatements_gbs": {k: round(v, 3) for k, v in both.items()}}
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
            "steps": K, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True,
            "scaling": "weak" if mode == "replicate" else "strong", "vs_baseline": None,
            "dtype": "bf16" if q.dtype == torch.bfloat16 else "f16", "data": "synthetic",
            "config": {"workload": w.name, "description": w.description, "mode": mode,
                       "num_seqs": w.num_seqs, "num_q_heads": w.num_q_heads,
                       "num_kv_heads": w.num_kv_heads, "head_size": w.head_size,
                       "block_size": w.block_size, "kv_bytes_per_step_all_gpus": total_bytes,
                       "kv_bytes_per_step_this_gpu": kv_bytes,
                       "parallelism": parallelism, "l2": l2_note},
            "us_per_call": round(ms_per_step * 1e3, 2),
            "hbm_frac_of_measured_peak": round(value / world / peak, 4),
            "gpu_launches_note": ("per step: planner, decode"
                                  + (", reduce" if launches == 3 else "")
                                  + ((", fused state exchange + merge" if exchange is not None
                                      else ", state merge (+ NCCL all-gather)")
                                     if mode == "split" else "")),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic, "peak_source": peak_src,
                         "kernel": "pab::decode_kernel", "kernel_us": round(kernel_ms * 1e3, 2),
                         "algorithmic_bytes_per_launch": kv_bytes,
                         "extra_bytes_per_call": extra_bytes,
                         "datasheet_peak": DATASHEET_HBM_GBS,
                         "datasheet_frac": round(achieved / DATASHEET_HBM_GBS, 4),
                         "traffic_source": traffic_src},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": E,
                    "note": "public in-place call (paged_attention / decode_context_parallel) "
                            "into two preallocated outputs; every step copies q, cache_seqlens "
                            "and block_table H2D from one pinned staging buffer in one copy (a "
                            "copy stream, two device buffers) and its output D2H; KV cache "
                            "resident"},
            "clocks": sampler.summary(),
            "graph": graph_line,
            "gpu_launches": (launches + (1 if mode == "split" else 0)) * K,
        }
    if world > 1:
        barrier()
        dist.destroy_process_group()
    if line is not None:
        emit(line)


_json_out = None


def emit(line: dict) -> None:
    """Write the one JSON result line to the process's original stdout."""
    out = _json_out or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    global _json_out
    # Libraries (NCCL, PyTorch) may print to stdout; keep stdout for the
    # single JSON line by pointing file descriptor 1 at stderr.
    sys.stdout.flush()
    _json_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
