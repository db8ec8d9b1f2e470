#!/usr/bin/env python
"""Benchmark of the fused spacetime-bias attention op (fwd + bwd) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload config1|config2|config3|config4] [--coords raw|scaled]
                    [--dim Dh --channels C --dtype bf16|fp16]   (config2)

One step is one forward + backward of the op through its public API
(``flash_spacetime_attention`` / ``..._varlen``) over one batch of seeded
synthetic events. The default workload is configuration 1 of the baseline:
B=256 events padded to L=768, H=12, Dh=32, C=16, bf16, lognormal lengths
(median 120, sigma 1.2 -- the sigma the baseline leaves open -- clipped to
[1, 768]). Throughput is algorithmic TFLOP/s over VALID pairs,
sum_b L_b^2 * H * (14 Dh + 12 C).

Other workloads: ``config2`` (B=128 full-length events of L=1024, H=8, the
``--dim``/``--channels``/``--dtype`` given), ``config3`` (16384 packed
lognormal events, median 80, 2 % single pulses) and ``config4`` (2048 packed
events of length uniform in [2048, 16384], strong scaling).

Under torchrun (N > 1) every rank owns a shard of the events chosen by
longest-first L^2 balancing: N x 256 events for config1 (weak scaling:
per-GPU work stays fixed), the fixed 2048 events of config4 (strong
scaling). Inside the step the per-rank dW/db partials are gathered and
summed the same way on every rank; for config4 (and with ``--gather-out``) the outputs
of all ranks are also all-gathered over NCCL after the backward (valid rows,
packed), as the sharded long-event run specifies. The step time is the max
over ranks of the device-timed duration.

Printed: one JSON line on rank 0 (see the keys below). ``value`` has inputs
resident in HBM; ``e2e`` repeats the step with the inputs copied from pinned
host memory and dW read back every step. ``--impl reference`` times the CPU
restatement of the upstream eager path (oracle/) on the host cores.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "flash-spacetime_b200"), ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

HEADS, DIM, CHANNELS = 12, 32, 16
METRIC = "fwd+bwd TFLOP/s (B=256,L=768,H=12,Dh=32,C=16 bf16; valid pairs)"


def _shape(args):
    """(heads, head dim, channels, dtype name, metric) of the workload."""
    if args.workload == "config2":
        d, c = args.dim or 32, args.channels or 32
        return 8, d, c, args.dtype, (f"fwd+bwd TFLOP/s (B=128,L=1024,H=8,Dh={d},C={c} "
                                     f"{args.dtype}; valid pairs)")
    if args.workload == "config1":
        return HEADS, DIM, CHANNELS, "bf16", METRIC
    desc = {"config3": "16384 packed events, lognormal median 80",
            "config4": "2048 packed events, L~U[2048,16384]"}[args.workload]
    return HEADS, DIM, CHANNELS, "bf16", f"fwd+bwd TFLOP/s ({desc}, H=12,Dh=32,C=16 bf16; valid pairs)"


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"bf16_tflops": float(d["bf16_tflops"]), "hbm_gbs": float(d["hbm_gbs"]),
                "src": "measured"}
    except Exception:
        return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0, "src": "fallback"}


def _traffic(workload: str):
    """DRAM bytes per launch of fst_forward / fst_backward from the committed
    ncu summary of this workload (profiles/dram_traffic_<workload>.txt), or {}."""
    path = os.path.join(ROOT, "profiles", f"dram_traffic_{workload}.txt")
    out = {}
    try:
        with open(path) as f:
            for line in f:
                line = line.strip()
                if line and not line.startswith("#") and "=" in line:
                    k, v = line.split("=", 1)
                    out[k] = v
    except OSError:
        return {}
    return out if out.get("workload") == workload else {}


def _dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _workload_lengths(name: str, world: int, rank: int, seed: int, events: int = 0):
    """(lengths of this rank's shard, padded length or None, global event
    count, every rank's shard lengths)."""
    from flash_spacetime.sharding import lpt_partition
    from flash_spacetime.synthetic import lengths_for

    if name == "config1":
        lens, padlen = lengths_for("config1", (events or 256) * world, seed), 768
    elif name == "config2":
        lens, padlen = [1024] * (128 * world), 1024
    elif name == "config3":
        lens, padlen = lengths_for("config3", 16384 * world, seed), None
    elif name == "config4":
        lens, padlen = lengths_for("config4", 2048, seed), None  # fixed total: strong scaling
    else:
        raise SystemExit(f"unknown workload {name}")
    shards = lpt_partition(lens, world) if world > 1 else [list(range(len(lens)))]
    per_rank = [[lens[i] for i in sh] for sh in shards]
    return per_rank[rank], padlen, len(lens), per_rank


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons; stop() keeps the samples
    whose timestamps fall inside the timed region."""

    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        import threading
        self.proc = None
        self.lines = []
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ident, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            # Drain the pipe as samples arrive: a long run fills the pipe's
            # buffer otherwise, and nvidia-smi stops sampling.
            self.reader = threading.Thread(target=self._drain, daemon=True)
            self.reader.start()
        except Exception:
            self.proc = None

    def _drain(self):
        for line in self.proc.stdout:
            self.lines.append(line)

    def stop(self, t0: float, t1: float):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
            self.reader.join(timeout=10)
        except Exception:
            self.proc.kill()
        out = "".join(self.lines)
        import datetime
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        samples = []
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                samples.append((ts, float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        inside = [x for x in samples if t0 - 0.06 <= x[0] <= t1 + 0.06]
        window = "timed region"
        if not inside:
            inside, window = samples[-3:], "last samples before stop (timed region shorter than the sampling period)"
        reasons = sorted({nm for x in inside for nm, flag in zip(names, x[3])
                          if flag.lower() == "active"})
        return {"sm_mhz": statistics.median([x[1] for x in inside]) if inside else None,
                "sm_max_mhz": max([x[2] for x in inside]) if inside else None,
                "samples": len(inside), "window": window, "reasons": reasons}


def cpu_eager_sample(lengths, budget_s: float, seed: int, heads: int = HEADS, dim: int = DIM,
                     channels: int = CHANNELS):
    """Time the CPU restatement of the upstream eager op, event by event.

    Runs fp32 forward + backward through autograd (upstream
    src/flash_spacetime/reference.py:106-167) on events of the workload in
    their natural order, passing over the workload again if needed, until
    ``budget_s`` seconds are spent; returns the achieved algorithmic TFLOP/s
    over the events done.
    """
    from oracle.spacetime_oracle import eager_fwd_bwd_fp32
    from flash_spacetime.synthetic import detector_coords, projection

    gen = torch.Generator().manual_seed(seed)
    proj = projection(dim, channels, gen)
    done_flops = 0.0
    done_pairs = 0
    spent = 0.0
    events = 0
    while spent < budget_s and len(lengths) > 0:
        for n in lengths:
            n = int(n)
            feats = detector_coords([n], gen).view(1, n, 4)
            q, k, v = (torch.randn(1, heads, n, dim, generator=gen) for _ in range(3))
            t0 = time.perf_counter()
            eager_fwd_bwd_fp32(q, k, v, feats, proj["weight"], proj["bias"], None)
            spent += time.perf_counter() - t0
            done_flops += n * n * heads * (14 * dim + 12 * channels)
            done_pairs += n * n
            events += 1
            if spent >= budget_s:
                break
    return {"tflops": done_flops / spent / 1e12 if spent > 0 else 0.0, "seconds": spent,
            "events": events, "pairs": done_pairs}


def run_reference(args):
    world, rank, _ = _dist_setup()
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    lens, _, _, _ = _workload_lengths(args.workload, 1, 0, args.seed)
    heads, dim, channels, _, metric = _shape(args)
    # Each step: a bounded sample of the workload's events (in order).
    for _ in range(args.warmup):
        cpu_eager_sample(lens, 0.5, args.seed, heads, dim, channels)
    vals, secs = [], []
    sample = None
    # Bounded per step so that the whole run stays near a minute and a half.
    budget = max(0.5, min(args.ref_budget, 90.0 / max(1, args.steps)))
    for _ in range(args.steps):
        sample = cpu_eager_sample(lens, budget, args.seed, heads, dim, channels)
        vals.append(sample["tflops"])
        secs.append(sample["seconds"])
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": metric, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * statistics.median(secs), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": args.workload, "events_per_step": sample["events"],
                   "pairs_per_step": sample["pairs"]},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"{sample['events']} events of {args.workload} in order "
                                   f"per step ({budget:.1f} s bounded), one event at a time, "
                                   "fp32 eager fwd+bwd via autograd"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_e2e(args, data, index, step, device, world, total_flops, lens, padded, expect,
            dim=DIM, channels=CHANNELS):
    """The step through the public API with every input copied from pinned
    host memory inside the timed region and dW/db read back each step.

    As a training loop's data loader would, the copy of step i+1's inputs is
    issued on a side stream while step i computes (two device slots, ordered
    by events); every step's own host->device copy is inside the timed region.
    A padded batch ships only its valid rows (``upload_valid_rows``, a gather
    kernel reading the pinned host rows; the kernels never read a padding
    row). The
    last step's dW/db must equal ``expect`` (the device-resident run's) bit
    for bit.
    """
    from flash_spacetime import ops
    from flash_spacetime.sharding import max_over_ranks

    keys = ("q", "k", "v", "grad", "feats", "weight", "bias")
    host = {k: data[k].detach().cpu().pin_memory() for k in keys}
    host["index"] = index.cpu().pin_memory()
    rows = ("q", "k", "v", "grad", "feats") if padded else ()
    h2d = 0
    for k, t in host.items():
        if k in rows:  # [B, H, L, D] or [B, L, 4]: sum(lens) rows of numel / (B L) elements
            length = t.shape[2] if t.dim() == 4 else t.shape[1]
            h2d += sum(lens) * (t.numel() // (t.shape[0] * length)) * t.element_size()
        else:
            h2d += t.numel() * t.element_size()
    dw_host = torch.empty(dim * channels + dim, dtype=torch.float32).pin_memory()
    d2h = dw_host.numel() * dw_host.element_size()

    slots = [{k: torch.zeros_like(t, device=device) for k, t in host.items()} for _ in range(2)]
    # High priority: the gather's few CTAs are placed as soon as an SM has
    # room instead of queueing behind the attention kernels' grid (4.06 vs
    # 4.45 ms per step on config 1).
    copy_stream = torch.cuda.Stream(device, priority=-1)
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    for ev in free:
        ev.record()

    def issue_copy(slot):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[slot])  # the step that used this slot is done
            for k, t in host.items():
                if k in rows:
                    ops.upload_valid_rows(slots[slot][k], t, lens)
                else:
                    slots[slot][k].copy_(t, non_blocking=True)
            ready[slot].record(copy_stream)

    def run(n):
        copy_stream.wait_stream(torch.cuda.current_stream())  # after the start event
        issue_copy(0)
        for i in range(n):
            slot = i % 2
            if i + 1 < n:
                issue_copy(1 - slot)
            torch.cuda.current_stream().wait_event(ready[slot])
            buf = slots[slot]
            lv = {k: buf[k].detach().requires_grad_(True)
                  for k in ("q", "k", "v", "weight", "bias")}
            # The next step's upload runs beside this step on every SM.
            _, dw, db = step(lv, buf["feats"], buf["grad"], buf["index"], share_sms=True)
            dw_host.copy_(torch.cat([dw.flatten().float(), db.flatten().float()]),
                          non_blocking=True)
            free[slot].record()

    run(max(1, args.warmup))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    run(args.steps)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, device)
    if not torch.equal(dw_host, expect.cpu()):
        raise RuntimeError("e2e: dW/db differ from the device-resident run")
    return {"value": total_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
            "overlap": "next step's host->device copy on a side stream (share_sms hint)",
            "transfer": ("valid rows only (upload_valid_rows: gather kernel reading pinned "
                         "host memory)" if padded else "whole tensors")}


def run_ours(args):
    world, rank, local = _dist_setup()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=device,
                                timeout=__import__("datetime").timedelta(seconds=120))
    from flash_spacetime import _lib, ops, synthetic
    from flash_spacetime.sharding import RowGather, gather_over_ranks, ordered_sum

    lens, padlen, n_events, per_rank = _workload_lengths(args.workload, world, rank, args.seed,
                                                         args.events)
    heads, dim, channels, dtype_name, metric = _shape(args)
    dtype = {"bf16": torch.bfloat16, "fp16": torch.float16}[dtype_name]
    scaled = args.coords == "scaled"
    if padlen is not None:
        data = synthetic.padded_batch(lens, padlen, heads, dim, channels, dtype, device,
                                      args.seed + 17 * rank, scaled)
    else:
        data = synthetic.packed_batch(lens, heads, dim, channels, dtype, device,
                                      args.seed + 17 * rank, scaled)
    # The generators' fp32 temporaries leave the caching allocator fragmented;
    # config4 needs ~150 GB of one GPU's memory in large blocks.
    torch.cuda.empty_cache()
    flops = synthetic.pair_flops(lens, heads, dim, channels)
    total_flops = sum(synthetic.pair_flops(x, heads, dim, channels)["total"] for x in per_rank)

    # The data tensors themselves are the leaves (no copies: config4 holds
    # 14 GB per [T, H, Dh] tensor on one GPU).
    leaves = {k: data[k].detach().requires_grad_(True) for k in ("q", "k", "v", "weight", "bias")}
    grad = data["grad"]
    feats = data["feats"]

    # Output all-gather across ranks: every rank's valid output rows, packed
    # ([rows, Dh]; a padded batch's valid rows are gathered by a precomputed
    # index), with the row counts known on every rank from the partition.
    gather = None
    want_gather = args.gather_out if args.gather_out is not None else args.workload == "config4"
    if world > 1 and want_gather:
        if padlen is not None:
            sizes = [sum(x) * heads for x in per_rank]
            idx = torch.cat([(b * heads + h) * padlen + torch.arange(n)
                             for b, n in enumerate(lens) for h in range(heads)]).to(device)
        else:
            sizes = [sum(x) * heads for x in per_rank]
            idx = None
        gather = RowGather(sizes, (dim,), dtype, device)
    gather_timer = [] if gather is not None else None

    # A data loader knows its batch's lengths on the host: passing their sum
    # lets the kernels launch blocks for the valid rows only.
    valid_rows = None if (padlen is None or args.full_grid) else sum(lens)

    def step(lv, feats_, grad_, seq_or_cu, share_sms=False):
        for t in lv.values():
            t.grad = None
        if padlen is not None:
            out = ops.flash_spacetime_attention(lv["q"], lv["k"], lv["v"], feats_, lv["weight"],
                                                lv["bias"], seq_or_cu, share_sms=share_sms,
                                                valid_rows=valid_rows)
        else:
            out = ops.flash_spacetime_attention_varlen(lv["q"], lv["k"], lv["v"], feats_,
                                                       lv["weight"], lv["bias"], seq_or_cu,
                                                       share_sms=share_sms)
        out.backward(grad_)
        if gather is not None:
            if gather_timer is not None:
                g0 = torch.cuda.Event(enable_timing=True)
                g0.record()
            # After the backward, not overlapping it: NCCL's kernels wait on
            # their peers while holding SMs, and next to the backward's SM-
            # filling kernels that cost 0.42 ms a step on 2 GPUs instead of
            # the ~0.1 ms the transfer takes on its own.
            rows = out.detach().view(-1, dim)
            n = gather.sizes[rank]
            if idx is not None:
                torch.index_select(rows, 0, idx, out=gather.send[:n])
            else:
                gather.send[:n].copy_(rows)
            gather.start().wait()
            if gather_timer is not None:
                g1 = torch.cuda.Event(enable_timing=True)
                g1.record()
                gather_timer.append((g0, g1))
        dw = lv["weight"].grad
        db = lv["bias"].grad
        if world > 1:
            flat = torch.cat([dw.flatten(), db.flatten()])
            flat = ordered_sum(flat)
            dw = flat[: dw.numel()].view_as(dw)
            db = flat[dw.numel():]
        return out, dw, db

    index = data["seqlens"] if padlen is not None else data["cu_seqlens"]
    timers = []
    ops.set_kernel_timer(timers)
    clocks = ClockSampler(local)  # started early so it is sampling by the timed region
    for _ in range(args.warmup):
        step(leaves, feats, grad, index)
    torch.cuda.synchronize()
    timers.clear()
    if gather_timer is not None:
        gather_timer.clear()

    torch.cuda.reset_peak_memory_stats(device)
    base_mem = torch.cuda.memory_allocated(device)
    lib = _lib.load()
    launches0 = lib.fst_kernel_launches()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    wall0 = time.time()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        _, dw_last, db_last = step(leaves, feats, grad, index)
    ev1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    wall1 = time.time()
    clk = clocks.stop(wall0, wall1)
    launches = lib.fst_kernel_launches() - launches0
    ms_local = ev0.elapsed_time(ev1) / args.steps
    ms = max(gather_over_ranks(ms_local, device))  # the slowest rank's step
    loads = [sum(n * n for n in x) for x in per_rank]
    peak_gib = (torch.cuda.max_memory_allocated(device) - base_mem) / 2**30
    ops.set_kernel_timer(None)

    # Per-kernel device times inside the timed steps.
    per = {}
    for name, e0, e1 in timers:
        per.setdefault(name, []).append(e0.elapsed_time(e1))
    gather_ms = (statistics.mean(a.elapsed_time(b) for a, b in gather_timer)
                 if gather_timer else None)
    fwd_ms = statistics.mean(per.get("fst_forward", [0.0]))
    bwd_ms = statistics.mean(per.get("fst_backward", [0.0]))
    # Every rank's attention kernels per step (the step times themselves are
    # equal across ranks: the dW / db all-gather waits for the slowest).
    rank_kernel_ms = gather_over_ranks(
        sum(statistics.mean(v) for v in per.values() if v), device)
    value = total_flops / (ms * 1e-3) / 1e12

    # End to end: inputs from pinned host memory every step, dW read back.
    e2e = None
    in_bytes = sum(data[k].numel() * data[k].element_size() for k in ("q", "k", "v", "grad"))
    if in_bytes > 16e9 and not args.no_e2e:
        e2e = {"skipped": f"inputs of {in_bytes / 1e9:.0f} GB per GPU exceed the pinned "
                          "host buffers this run allocates (16 GB)"}
    elif not args.no_e2e:
        expect = torch.cat([dw_last.flatten().float(), db_last.flatten().float()])
        e2e = run_e2e(args, data, index, step, device, world, total_flops, lens,
                      padlen is not None, expect, dim, channels)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks = _peaks()
    dom = "fst_backward" if bwd_ms >= fwd_ms else "fst_forward"
    dom_ms = bwd_ms if dom == "fst_backward" else fwd_ms
    dom_flops = flops["bwd"] if dom == "fst_backward" else flops["fwd"]
    achieved = dom_flops / (dom_ms * 1e-3) / 1e12 if dom_ms > 0 else 0.0
    tr = _traffic(args.workload) if args.coords == "raw" and world == 1 else {}
    traffic = int(tr[dom]) if dom in tr else None

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        s = cpu_eager_sample(lens, args.cpu_budget, args.seed, heads, dim, channels)
        cpu = {"value": s["tflops"], "unit": "TFLOP/s", "cores": torch.get_num_threads(),
               "kind": "port",
               "sample": f"{s['events']} events ({s['pairs']} valid pairs) of "
                         f"{args.workload} in order (repeating the workload), one event at "
                         f"a time, fp32 eager fwd+bwd via autograd, {s['seconds']:.1f} s"}

    line = {
        "metric": metric, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak" if args.workload != "config4" else "strong",
        "vs_baseline": None, "dtype": dtype_name, "data": "synthetic",
        "config": {"workload": args.workload, "events": n_events, "heads": heads,
                   "head_dim": dim, "channels": channels,
                   "padded_length": padlen, "coords": args.coords,
                   "valid_rows_hint": valid_rows,
                   "valid_pairs_per_gpu": flops["pairs"],
                   "output_gather": (None if gather is None else
                                     f"all_gather_into_tensor of every rank's valid output rows, "
                                     f"{gather.bytes_received() / 1e6:.0f} MB received per rank "
                                     f"per step, after the backward"),
                   "l2_policy": f"inputs larger than L2 (q, k, v, grad "
                                f"{data['q'].numel() * data['q'].element_size() / 1e6:.0f} MB "
                                f"each)"},
        "fwd_ms": fwd_ms, "bwd_ms": bwd_ms, "gather_ms": gather_ms, "peak_gib": peak_gib,
        # Per valid (query, key) pair, as the kernels evaluate them: each of
        # the three kernels (forward, row, column) forms E_ij once for all
        # heads (C/2 sin + C/2 cos after one shared range reduction) and the
        # interval's sqrt once, and one exp2 per head.
        "transcendentals_per_pair": {"sin_cos": 3 * channels, "sqrt": 3, "exp2": 3 * heads,
                                     "total": 3 * (channels + 1 + heads)},
        "roofline": {"bound": "tensor", "kernel": dom, "achieved": achieved,
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16_tflops"], "traffic": traffic,
                     "traffic_unit": "bytes per launch (ncu dram read + write)",
                     "peak_src": peaks["src"] + " burst bf16"},
        "cpu_baseline": cpu,
        "clocks": clk,
        "e2e": e2e,
        "gpu_launches": launches,
        # Per-rank library kernel time a step (forward, backward and the dW /
        # db sums) and the partition's balance of valid pairs (the sharding
        # key): the job's step is the slowest rank's.
        "ranks": {"kernel_ms_min": min(rank_kernel_ms), "kernel_ms_max": max(rank_kernel_ms),
                  "kernel_ms_mean": sum(rank_kernel_ms) / len(rank_kernel_ms),
                  "pairs_max_over_mean": max(loads) / (sum(loads) / len(loads))},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default="config1",
                    choices=("config1", "config2", "config3", "config4"))
    ap.add_argument("--dim", type=int, default=0, help="config2 head dim (32 or 64)")
    ap.add_argument("--channels", type=int, default=0, help="config2 channels (32 or 64)")
    ap.add_argument("--dtype", default="bf16", choices=("bf16", "fp16"), help="config2 dtype")
    ap.add_argument("--events", type=int, default=0,
                    help="config1 events per GPU (default 256; smaller for profiler captures)")
    ap.add_argument("--gather-out", dest="gather_out", action="store_true", default=None,
                    help="multi-GPU: all-gather every rank's outputs inside the step "
                         "(the default for config4, whose sharded run names it)")
    ap.add_argument("--no-gather", dest="gather_out", action="store_false",
                    help="multi-GPU: skip the all-gather of the outputs")
    ap.add_argument("--full-grid", action="store_true",
                    help="padded workloads: do not pass the valid row count (valid_rows), so "
                         "the kernels launch blocks over all B x L rows")
    ap.add_argument("--coords", default="raw", choices=("raw", "scaled"))
    ap.add_argument("--seed", type=int, default=2026)
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--ref-budget", type=float, default=6.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the host-buffer pass (for profiler runs)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "config4":
        # ~150 GB of one GPU in large blocks that are freed and re-taken every
        # step; expandable segments keep the caching allocator from
        # fragmenting (read when CUDA initialises, which has not happened yet).
        os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
