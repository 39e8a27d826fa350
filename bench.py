"""Benchmark: paged-attention decode µs/call and KV-read TB/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c5] [--impl ours|reference]

One step = one decode call over one batch of the workload, inputs resident
in HBM.  Default workload c5 (the 1/2/4/8-GPU serving batch of the spec:
256 sequences, 64/8 heads, lengths U[1,32768] with 5% empty, fp16, vLLM
layout, 16 GB of KV); at N GPUs (torchrun, one rank per GPU) every rank owns
8/N KV heads and their pages, so total work is fixed ("strong" scaling).
Other workloads (c1..c4) are available with --workload.

Printed (rank 0, one JSON line): value = aggregate KV-read TB/s over all
ranks (KV bytes of the whole batch / max-over-ranks device time), the
µs/call, the roofline of the partition kernel against the measured HBM
copy bandwidth, the CPU baseline (the oracle's C port on this host's cores,
bounded sample), the end-to-end number through the public API with pinned
host buffers, clocks sampled by NVML during the timed region, and the number
of this library's kernel launches in the timed region.

--impl reference times the reference's CPU implementation (restated by the
oracle's multithreaded C port; the reference has no other CPU path) on a
bounded sample of the same workload on this host's cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "paged-attn decode KV-read TB/s (µs/call; % HBM peak) at N B200"
UNIT = "TB/s"


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def _profile_traffic(workload: str) -> float | None:
    """Per-launch DRAM bytes of the partition kernel from the committed ncu summary, if any."""
    p = ROOT / "profiles" / f"traffic_{workload}.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["dram_bytes_per_launch"])
        except (KeyError, ValueError):
            return None
    return None


class ClockSampler:
    """NVML sampling of SM clocks and throttle reasons in a background thread."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clocks_setting": 0x100,
    }

    def __init__(self, indices, interval=0.01):
        self.samples = []
        self.interval = interval
        self._stop = threading.Event()
        self._thread = None
        self.max_mhz = None
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handles = [pynvml.nvmlDeviceGetHandleByIndex(i) for i in indices]
            self.max_mhz = max(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM) for h in self._handles)
            self.ok = True
        except Exception as e:  # noqa: BLE001
            self.error = str(e)

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            for h in self._handles:
                try:
                    mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((time.perf_counter(), mhz, int(reasons)))
                except Exception:  # noqa: BLE001
                    pass
            time.sleep(self.interval)

    def start(self):
        if self.ok:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self):
        if self._thread:
            self._stop.set()
            self._thread.join()

    def summary(self, t0, t1) -> dict:
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "note": "NVML unavailable"}
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        used = inside if inside else self.samples[-3:]
        reasons = set()
        for _, _, r in used:
            for name, bit in self.REASONS.items():
                if r & bit and name != "gpu_idle":
                    reasons.add(name)
        mhz = statistics.median(s[1] for s in used) if used else None
        out = {"sm_mhz": mhz, "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons), "samples": len(inside)}
        if not inside:
            out["note"] = "timed region shorter than the sampling interval; nearest samples used"
        return out


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, ws, local


# ---------------------------------------------------------------------------
# CPU (reference) arm
# ---------------------------------------------------------------------------
def _cpu_sample(workload: str, target_bytes: float):
    """Sequences of the workload (chosen by a seeded draw over the non-empty
    ones) adding up to ~target_bytes of KV, materialised on the host."""
    import torch

    from decodekernels_b200 import workloads

    lens = workloads.seq_lens(workload)
    c = workloads.CONFIGS[workload]
    per_tok = c.num_kv_heads * c.head_dim * 2 * c.kv_bytes_per_elem
    order = torch.randperm(len(lens), generator=torch.Generator().manual_seed(11)).tolist()
    chosen, total = [], 0
    for i in order:
        if lens[i] <= 0:
            continue
        chosen.append(i)
        total += lens[i] * per_tok
        if total >= target_bytes:
            break
    batch = workloads.make(workload, "cpu", seqs=sorted(chosen))
    return batch


def workloads_dequantize(batch):
    """A CPU sample's cache as 16-bit values (e4m3 configs: code * scale,
    exact), for the 16-bit C oracle."""
    from decodekernels_b200 import workloads

    return workloads.dequantize(batch.kv, batch.config)


def workloads_lens(workload: str) -> list[int]:
    from decodekernels_b200 import workloads

    return workloads.seq_lens(workload)


def cpu_throughput(workload: str, seconds: float, target_bytes: float = 256e6, steps: int | None = None,
                   warmup: int = 0):
    """Time the oracle's C port (all host threads) on a bounded sample."""
    from oracle import native

    b = _cpu_sample(workload, target_bytes)
    kv = workloads_dequantize(b)
    args = (b.q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
    for _ in range(warmup):
        native.dense_c(*args)
    times = []
    t_end = time.perf_counter() + seconds
    while (steps is None and (time.perf_counter() < t_end or not times)) or (steps is not None and len(times) < steps):
        t = time.perf_counter()
        native.dense_c(*args)
        times.append(time.perf_counter() - t)
    per_call = statistics.median(times)
    kvb = b.kv_bytes()
    return {
        "value": kvb / per_call / 1e12,
        "unit": UNIT,
        "cores": native.max_threads(),
        "kind": "port",
        "sample": f"{len(b.lens)} of {len(workloads_lens(workload))} sequences of {workload} "
                  f"({sum(b.lens)} tokens, {kvb / 1e6:.0f} MB KV), median of {len(times)} calls of the oracle's "
                  f"C port (OpenMP, all host threads)" + (" on the caches dequantised to 16 bits (the reference "
                                                          "has no e4m3 path)" if b.config.kv_fp8 else ""),
        "seconds_per_call": per_call,
        "calls": len(times),
    }


def run_reference_arm(args) -> None:
    rank, world, _ = _dist()
    if rank != 0:
        return
    from oracle import build as obuild

    obuild.build_oracle()
    # each step is one oracle call over a ~64 MB sample so K + W steps stay within minutes
    res = cpu_throughput(args.workload, 0, target_bytes=64e6, steps=args.steps, warmup=args.warmup)
    v = res["value"]
    line = {
        "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["seconds_per_call"] * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": args.workload, "sample": res["sample"]},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": res["cores"], "kind": "port", "sample": res["sample"]},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def _check_parity(batch, out, rank) -> dict:
    """Compare a few sequences of the call's output with the C oracle."""
    import numpy as np

    from decodekernels_b200 import workloads
    from oracle import native

    lens = batch.lens
    live = [i for i, L in enumerate(lens) if L > 0]
    pick = sorted(set([live[0], max(live, key=lambda i: lens[i]), min(live, key=lambda i: lens[i])]
                      + [i for i, L in enumerate(lens) if L == 0][:1]))
    q, kv = workloads.compact_sequences(batch, pick)
    kv = workloads.dequantize(kv, batch.config)  # e4m3 configs: the exact 16-bit values of the codes
    ref = native.dense_c(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
    got = out[pick].float().cpu().numpy()
    err = np.abs(got - ref)
    ok = bool(np.isfinite(got).all() and err.max() <= 2e-2 and err.mean() <= 2e-3)
    if not ok:
        raise SystemExit(f"rank {rank}: parity check failed before timing (max-abs {err.max():.3e}, "
                         f"mean-abs {err.mean():.3e}) on sequences {pick}")
    return {"sequences": pick, "max_abs": float(err.max()), "mean_abs": float(err.mean())}


def run_gpu_arm(args) -> None:
    import torch

    rank, world, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    import decodekernels_b200 as dk
    from decodekernels_b200 import capi, workloads

    if not dk.is_available():
        raise SystemExit(f"decodekernels_b200 native library unavailable: {dk.ops._IMPORT_ERROR}")

    cfg = workloads.CONFIGS[args.workload]
    sharding = args.sharding
    if sharding == "auto":
        sharding = "head" if cfg.num_kv_heads % world == 0 else "seq"
    seq_mode = world > 1 and sharding == "seq"
    if seq_mode:
        # Sequence sharding: every rank holds its striped blocks of every
        # sequence and the whole query; a step is the rank's partials, one
        # NCCL all-gather of them and the log-sum-exp merge (full output on
        # every rank).
        from decodekernels_b200.sharded import SequenceShardedPagedAttention, striped_max_len

        batch = workloads.make_striped(args.workload, dev, stripe=(rank, world))
        seq_attn = SequenceShardedPagedAttention(block_size=batch.config.block_size, rank=rank, world=world,
                                                 exchange=args.exchange)
        full_max = max(workloads.seq_lens(args.workload))
        max_len = striped_max_len(full_max, batch.config.block_size, world)
    else:
        batch = workloads.make(args.workload, dev, shard=(rank, world))
        max_len = batch.max_seq_len
    q, kv = batch.q, batch.kv
    n, hq, d = q.shape
    out = torch.empty_like(q)
    ws = dk.alloc_workspace(n, hq, d, max_len, dev, num_kv_heads=kv.k_cache.shape[2],
                            block_size=kv.block_size, merge_counters=not seq_mode)
    fp8_scale = batch.config.kv_scale if batch.config.kv_fp8 else 1.0
    plan = capi.plan(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, d**-0.5, max_len, out, ws,
                     k_scale=fp8_scale, v_scale=fp8_scale)

    if seq_mode:
        def step():
            seq_attn(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, max_seq_len=full_max, out=out,
                     workspace=ws, k_scale=fp8_scale, v_scale=fp8_scale)
    else:
        kscale = batch.config.kv_scale if batch.config.kv_fp8 else 1.0

        def step():
            dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, max_seq_len=max_len,
                                      out=out, workspace=ws, k_scale=kscale, v_scale=kscale)

    step()
    torch.cuda.synchronize()
    parity = _check_parity(batch, out, rank) if not seq_mode else {
        "checked": "sequence-sharded merge parity is covered by tests/test_gpu_seq_sharded.py"}

    # Inputs several times the 126 MB L2 (c2-c5) stream through it with no
    # reuse between steps; smaller ones (c1) get a 256 MB write between steps.
    l2_bytes = 126 * 1024 * 1024
    flush = batch.kv_bytes() < 3 * l2_bytes
    flush_buf = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.int32, device=dev) if flush else None

    sampler = ClockSampler([local] if world == 1 else list(range(world))) if rank == 0 else None
    if sampler:
        sampler.start()

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        if flush:
            flush_buf.zero_()
        step()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.steps):
        if flush:
            flush_buf.zero_()
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    t1 = time.perf_counter()
    per_step = [s.elapsed_time(e) * 1e-3 for s, e in zip(starts, ends)]  # seconds, kernels only
    device_s = sum(per_step)
    if sampler:
        sampler.stop()

    # With N GPUs, also time the variant whose consumer needs every head on
    # every rank: decode + all-gather of the per-head outputs -- with
    # --exchange p2p the gather rides on the decode's output stores (peer
    # stores over NVLink, dk_paged_attention_decode_gather), with nccl an
    # all_gather_into_tensor follows the decode.
    gather_s = None
    gatherer = None
    if world > 1 and not seq_mode:
        from decodekernels_b200.sharded import ShardedPagedAttention

        gatherer = ShardedPagedAttention(batch.config.num_q_heads, batch.config.num_kv_heads, rank, world,
                                         exchange=args.exchange)
        full_out = torch.empty(out.shape[0], batch.config.num_q_heads, out.shape[2], dtype=out.dtype, device=dev)

        def gather_step():
            if args.exchange == "p2p" and not batch.config.kv_fp8:
                gatherer(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, max_seq_len=max_len,
                         workspace=ws, gather=True, gathered_out=full_out)
            else:
                step()
                gatherer.gather(out, full_out)

        for _ in range(3):
            gather_step()
        torch.cuda.synchronize()
        if not torch.equal(full_out[:, rank * out.shape[1]:(rank + 1) * out.shape[1]], out):
            raise SystemExit(f"rank {rank}: the gathered output's own heads differ from the decode's")
        torch.distributed.barrier()
        torch.cuda.synchronize()
        gs, ge = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        gs.record(stream)
        for _ in range(args.steps):
            gather_step()
        ge.record(stream)
        torch.cuda.synchronize()
        gather_s = gs.elapsed_time(ge) * 1e-3

    # End to end through the public API with pinned host buffers, as a serving
    # loop runs it: every step copies its inputs (q, block tables, lengths)
    # host -> device and reads its output back device -> host.  The copies run
    # on two copy streams (one per direction: PCIe is full duplex) into double
    # buffers, so step i + 1's inputs and step i - 1's output cross PCIe while
    # step i's decode runs; the timed window spans the first input copy to the
    # last output read.
    # A step's inputs sit in one pinned staging buffer (q | block tables |
    # lengths, each 256-byte aligned), as a serving loop prepares them, and
    # cross PCIe in one copy; the device tensors are views of its copy.
    parts = [q.contiguous(), kv.block_tables.contiguous(), kv.seq_lens.contiguous()]
    offs, total = [], 0
    for t in parts:
        offs.append(total)
        total += -(-t.numel() * t.element_size() // 256) * 256
    h_stage = torch.empty(total, dtype=torch.uint8, pin_memory=True)
    for t, o in zip(parts, offs):
        nb = t.numel() * t.element_size()
        h_stage[o:o + nb].copy_(t.view(-1).view(torch.uint8).cpu())
    h2d = total  # bytes copied per step (the staging buffer, alignment padding included)
    d2h = out.numel() * out.element_size()
    h2d_stream = torch.cuda.Stream(dev)
    d2h_stream = torch.cuda.Stream(dev)
    d_stage = [torch.empty(total, dtype=torch.uint8, device=dev) for _ in range(2)]

    def views(buf):
        return tuple(buf[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape) for t, o in zip(parts, offs))

    ins = [views(d_stage[b]) for b in range(2)]
    outs = [torch.empty_like(out) for _ in range(2)]
    h_outs = [torch.empty(out.shape, dtype=out.dtype, pin_memory=True) for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def h2d_copy(b):  # on the host -> device stream
        d_stage[b].copy_(h_stage, non_blocking=True)
        ev_in[b].record(h2d_stream)

    def decode(b):  # on the compute stream
        qd, btd, sld = ins[b]
        if seq_mode:
            seq_attn(qd, kv.k_cache, kv.v_cache, btd, sld, max_seq_len=full_max, out=outs[b], workspace=ws,
                     k_scale=fp8_scale, v_scale=fp8_scale)
        else:
            dk.paged_attention_decode(qd, kv.k_cache, kv.v_cache, btd, sld, max_seq_len=max_len, out=outs[b],
                                      workspace=ws, k_scale=kscale, v_scale=kscale)

    def e2e_run(nsteps, start_event=None):
        if start_event is not None:
            h2d_stream.wait_event(start_event)
            d2h_stream.wait_event(start_event)
        with torch.cuda.stream(h2d_stream):
            h2d_copy(0)
        for i in range(nsteps):
            b = i % 2
            stream.wait_event(ev_in[b])
            if i >= 2:
                stream.wait_event(ev_out[b])  # outs[b]'s previous read-back is done
            if flush:
                flush_buf.zero_()
            decode(b)
            ev_comp[b].record(stream)
            if i + 1 < nsteps:
                with torch.cuda.stream(h2d_stream):
                    if i >= 1:
                        h2d_stream.wait_event(ev_comp[1 - b])  # step i - 1 no longer reads those inputs
                    h2d_copy(1 - b)
            with torch.cuda.stream(d2h_stream):
                d2h_stream.wait_event(ev_comp[b])
                h_outs[b].copy_(outs[b], non_blocking=True)
                ev_out[b].record(d2h_stream)
        stream.wait_stream(h2d_stream)
        stream.wait_stream(d2h_stream)

    e2e_run(max(args.warmup, 3))
    e_steps = max(10, min(args.steps, 100))
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record(stream)
    e2e_run(e_steps, es)
    ee.record(stream)
    torch.cuda.synchronize()
    e2e_s = es.elapsed_time(ee) * 1e-3
    e2e_out, dev_out = h_outs[(e_steps - 1) % 2].float(), out.float().cpu()
    if not torch.equal(e2e_out, dev_out):
        diff = (e2e_out - dev_out).abs()
        raise SystemExit(f"rank {rank}: the end-to-end output differs from the device-timed call's: "
                         f"{int((diff > 0).sum())} elements, max {float(diff.nan_to_num(0.0).max()):.3e}, "
                         f"NaN {int(torch.isnan(e2e_out).sum())} / {int(torch.isnan(dev_out).sum())}")
    if flush:  # remove the flush time from the end-to-end window
        fs, fe = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        fs.record(stream)
        for _ in range(e_steps):
            flush_buf.zero_()
        fe.record(stream)
        torch.cuda.synchronize()
        e2e_s -= fs.elapsed_time(fe) * 1e-3

    kv_local = batch.kv_bytes()
    alg_local = batch.algorithmic_bytes()
    stats = torch.tensor([device_s, e2e_s, gather_s or 0.0, float(kv_local), float(alg_local)], dtype=torch.float64,
                         device=dev)
    if world > 1:
        import torch.distributed as dist

        tmax = stats[:3].clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        sums = stats[3:].clone()
        dist.all_reduce(sums, op=dist.ReduceOp.SUM)
        device_s, e2e_s, gather_s = tmax.tolist()
        kv_total, alg_total = sums.tolist()
    else:
        kv_total, alg_total = float(kv_local), float(alg_local)

    if rank == 0:
        step_s = device_s / args.steps
        value = kv_total / step_s / 1e12
        peaks = _peaks()
        # roofline of this rank's launches: algorithmic bytes per call / mean call time
        local_step = sum(per_step) / len(per_step)
        achieved = alg_local / local_step / 1e9
        traffic = _profile_traffic(args.workload) if world == 1 else None
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_s * 1e3, "us_per_call": step_s * 1e6,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": ("e4m3 KV, f16 mma" if batch.config.kv_fp8 else
                      ("f16" if batch.config.dtype == torch.float16 else "bf16")),
            "accumulate": "f32", "data": "synthetic",
            "impl": "ours",
            "config": {
                "workload": f"{args.workload}: {batch.config.description}",
                "num_seqs": n, "num_q_heads": batch.config.num_q_heads, "num_kv_heads": batch.config.num_kv_heads,
                "head_dim": d, "block_size": kv.block_size, "max_seq_len": max_len,
                "kv_bytes_total": kv_total, "algorithmic_bytes_total": alg_total,
                "parallelism": ((f"sequence shard (block-striped) x{world}, partials pushed to every GPU over "
                                 "NVLink peer memory + LSE merge in one kernel every step" if args.exchange == "p2p"
                                 else f"sequence shard (block-striped) x{world}, NCCL all-gather of partials + "
                                      "LSE merge in every step") if seq_mode else f"kv-head shard x{world}")
                               if world > 1 else "single GPU",
                "l2": "L2 flushed (256 MB write) before every step" if flush else
                      "inputs larger than L2 (no flush between steps)",
                "plan": plan, "parity": parity,
            },
            "roofline": {
                "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                "peak_source": f"{peaks['source']} HBM copy bandwidth",
                "note": "achieved = algorithmic bytes per call / CUDA-event time of the whole call "
                        "(partition + merge kernels)",
            },
            "e2e": {"value": kv_total / (e2e_s / e_steps) / 1e12, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e_steps, "api": "decodekernels_b200.paged_attention_decode",
                    "copies": "pinned host buffers; each step's inputs (q, block tables, lengths in one staging "
                              "buffer) H2D and its output D2H on one copy stream per direction, double buffered, "
                              "overlapping the neighbouring steps' decode"},
            "gpu_launches": args.steps * (plan["launches"] + (1 if seq_mode else 0)),
            "exchange_errors": (seq_attn.p2p_errors() if seq_mode
                                else gatherer.p2p_errors() if gatherer is not None else None),
            "with_gather": None if not gather_s else {
                "us_per_call": gather_s / args.steps * 1e6, "value": kv_total / (gather_s / args.steps) / 1e12,
                "unit": UNIT, "note": "decode + all-gather of the per-head outputs to every rank ("
                + ("NCCL)" if args.exchange != "p2p" else
                   "one NVLink peer-memory kernel after the decode, dk_gather_heads)" if batch.config.kv_fp8 else
                   "fused into the decode's output stores over NVLink peer memory, dk_paged_attention_decode_gather)")},
            "clocks": sampler.summary(t0, t1) if sampler else None,
            "wall_s_timed": t1 - t0,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_throughput(args.workload, seconds=args.cpu_seconds)
            line["cpu_baseline"].pop("calls", None)
        print(json.dumps(line), flush=True)

    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="c5",
                    choices=["c1", "c2", "c3", "c4", "c5", "c2f8", "c3f8", "c4f8", "c5f8"])
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="N>1: the collective over NVLink peer memory (one kernel of ours) or NCCL; sequence "
                         "sharding: the partial rows' exchange + merge, head sharding: the all-gather of the "
                         "per-head outputs timed beside the decode (with_gather)")
    ap.add_argument("--sharding", default="auto", choices=["auto", "head", "seq"],
                    help="N>1: KV-head sharding (no exchange) or block-striped sequence sharding (partials "
                         "all-gathered and merged every step); auto = head when the KV heads divide evenly")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    _, world, _ = _dist()
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}; using WORLD_SIZE", file=sys.stderr)
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_gpu_arm(args)


if __name__ == "__main__":
    main()
