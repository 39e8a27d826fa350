"""Benchmark: paged-attention decode µs/call and KV-read TB/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c5] [--impl ours|reference]

One step = one decode call over one batch of the workload, inputs resident
in HBM.  Default workload c5 (the 1/2/4/8-GPU serving batch of the spec:
256 sequences, 64/8 heads, lengths U[1,32768] with 5% empty, fp16, vLLM
layout, 16 GB of KV); at N GPUs (torchrun, one rank per GPU) every rank owns
8/N KV heads and their pages, so total work is fixed ("strong" scaling).
Other workloads (c1..c4, e4m3 variants) are available with --workload.

Printed (rank 0, one JSON line): value = aggregate KV-read TB/s over all
ranks (KV bytes of the whole batch / max-over-ranks device time of K
back-to-back calls), the µs/call, the roofline of the call against the
measured HBM copy bandwidth, the end-to-end number through the public API
with pinned host buffers, clocks sampled by NVML during the timed region, the
number of this library's kernel launches in the timed region, and:

* ``cpu_baseline`` (N=1): the reference's own CPU implementation
  (``decode_kernels.reference.paged_attention_reference``, PyTorch, from the
  reference installed into ``baseline/_ref``) on this host's cores over a
  bounded seeded sample of the workload, and the oracle's C port on the same
  sample;
* ``reference_kernel`` and ``also`` (N=1): the reference's CUDA kernel (built
  from its source for sm_100a) timed on the same device tensors the way the
  reference's benchmark times (10 warm-up calls, 100 calls each after a
  256 MB L2 flush, median), beside this library timed the same way, for the
  headline workload and for c2, c3, c4 and their e4m3 variants, and
  FlashInfer's batch decode (the reference benchmark's baseline) on c2-c4;
* ``gather_parity`` (N>1): every head of the gathered output (head sharding)
  or of the merged output (sequence sharding) on every rank checked against
  the CPU oracle on sample sequences.

--impl reference times the reference's CPU implementation only (no GPU, no
code of this library), on the same sample as ``cpu_baseline``; under
torchrun rank 0 runs it and the other ranks exit.
"""

from __future__ import annotations

import argparse
import importlib
import importlib.util
import json
import os
import statistics
import sys
import threading
import time
import types
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "paged-attn decode KV-read TB/s (µs/call; % HBM peak) at N B200"
UNIT = "TB/s"
L2_BYTES = 126 * 1024 * 1024
# Inputs above 1.5 x L2 are timed back to back without a flush: back-to-back
# launches of the e4m3 c2-c4 batches (200-320 MB) read 0.957-0.987 of their
# algorithmic bytes from DRAM (ncu), so little survives in L2 between calls,
# while a flush leaves L2 full of dirty lines that the next call writes back.
FLUSH_BELOW = 1.5 * L2_BYTES
CPU_SAMPLE_BYTES = 64e6  # KV bytes of the CPU sample (both arms time the same sample)
MAX_ABS, MEAN_ABS = 2e-2, 2e-3  # parity bounds for fp16 / bf16 outputs


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


def _sig(x: float, digits: int = 4) -> float:
    return float(f"{x:.{digits}g}")


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


def _usable_cores() -> int:
    """Host cores this process may run on (torchrun's OMP_NUM_THREADS=1 does not change it)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# Workload description shared by both arms
# ---------------------------------------------------------------------------
def _inputs():
    """The seeded input generator (decodekernels_b200/workloads.py and
    testing.py, plain PyTorch) loaded WITHOUT the package's __init__, which
    maps this library's native code: the reference arm and the CPU legs must
    not load it."""
    name = "_dkb_inputs"
    mod = sys.modules.get(name + ".workloads")
    if mod is None:
        pkg = types.ModuleType(name)
        pkg.__path__ = [str(ROOT / "decodekernels_b200")]
        sys.modules[name] = pkg
        mod = importlib.import_module(name + ".workloads")
    return mod


def _seq_mode(name: str, world: int, sharding: str) -> bool:
    w = _inputs()
    if sharding == "auto":
        sharding = "head" if w.CONFIGS[name].num_kv_heads % world == 0 else "seq"
    return world > 1 and sharding == "seq"


def workload_config(name: str, world: int, seq_mode: bool, exchange: str) -> dict:
    """The ``config`` object of the JSON line: the workload and how it is run,
    computed from the workload definition alone so both arms print the same."""
    w = _inputs()
    c = w.CONFIGS[name]
    lens = w.seq_lens(name)
    kv_total = sum(lens) * c.num_kv_heads * c.head_dim * 2 * c.kv_bytes_per_elem
    flush = kv_total / world < FLUSH_BELOW
    if world == 1:
        par = "single GPU"
    elif seq_mode:
        par = (f"sequence shard (block-striped) x{world}, partials pushed to every GPU over NVLink peer memory + "
               "LSE merge in one kernel every step" if exchange == "p2p" else
               f"sequence shard (block-striped) x{world}, NCCL all-gather of partials + LSE merge in every step")
    else:
        par = f"kv-head shard x{world}"
    return {
        "workload": f"{name}: {c.description}",
        "num_seqs": c.num_seqs, "num_q_heads": c.num_q_heads, "num_kv_heads": c.num_kv_heads,
        "head_dim": c.head_dim, "block_size": c.block_size, "max_seq_len": max(lens), "kv_bytes_total": kv_total,
        "parallelism": par,
        "l2": "L2 flushed (256 MB write) before every step" if flush else "inputs larger than L2 (no flush between steps)",
    }


# ---------------------------------------------------------------------------
# CPU legs: the reference's CPU implementation and the oracle's C port
# ---------------------------------------------------------------------------
def _cpu_sample(name: str, target_bytes: float = CPU_SAMPLE_BYTES):
    """Sequences of the workload (a seeded draw over the non-empty ones)
    adding up to ~target_bytes of KV, materialised on the host; e4m3 caches
    dequantised to 16 bits (exact: code x power-of-two scale), since the
    reference has no e4m3 path."""
    import torch

    w = _inputs()
    lens = w.seq_lens(name)
    c = w.CONFIGS[name]
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
    batch = w.make(name, "cpu", seqs=sorted(chosen))
    kv = w.dequantize(batch.kv, batch.config)
    desc = (f"{len(batch.lens)} of {len(lens)} sequences of {name} ({sum(batch.lens)} tokens, "
            f"{batch.kv_bytes() / 1e6:.0f} MB KV)" + (", e4m3 caches dequantised to 16 bits" if c.kv_fp8 else ""))
    return batch, kv, desc


def _reference_cpu_fn():
    """``paged_attention_reference`` from the reference's own package as
    installed into baseline/_ref (unmodified; loaded by file so that this
    repository's ``decode_kernels`` package of the same name does not shadow
    it, and without the reference's CUDA extension, which the CPU path does
    not use).  None when it is not installed."""
    p = ROOT / "baseline" / "_ref" / "decode_kernels" / "reference.py"
    if not p.exists():
        return None
    spec = importlib.util.spec_from_file_location("_dk_reference_cpu", p)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.paged_attention_reference


def _time_calls(fn, steps=None, warmup=0, seconds=None):
    for _ in range(warmup):
        fn()
    times = []
    t_end = time.perf_counter() + (seconds or 0.0)
    while (len(times) < steps) if steps is not None else (time.perf_counter() < t_end or len(times) < 3):
        t = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t)
    return times


def cpu_measure(name: str, steps=None, warmup=0, seconds=None) -> dict:
    """Time the reference's CPU implementation (when installed) and the
    oracle's C port on the same sample, with every usable host core."""
    import torch

    batch, kv, desc = _cpu_sample(name)
    cores = _usable_cores()
    args = (batch.q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
    kvb = batch.kv_bytes()
    res = {}
    ref_fn = _reference_cpu_fn()
    if ref_fn is not None:
        torch.set_num_threads(cores)
        times = _time_calls(lambda: ref_fn(*args), steps, warmup, seconds)
        res["reference"] = {
            "value": kvb / statistics.median(times) / 1e12, "unit": UNIT, "cores": torch.get_num_threads(),
            "cores_asked": cores, "kind": "reference", "seconds_per_call": statistics.median(times),
            "calls": len(times),
            "sample": f"{desc}; median of {len(times)} calls of the reference's "
                      "decode_kernels.reference.paged_attention_reference (PyTorch CPU, torch threads = usable "
                      "cores), installed unmodified into baseline/_ref"}
    from oracle import build as obuild
    from oracle import native

    obuild.build_oracle()
    info = {}
    port_seconds = seconds if ref_fn is None or seconds is None else seconds / 2
    times = _time_calls(lambda: native.dense_c(*args, num_threads=cores, info=info), steps, warmup, port_seconds)
    res["port"] = {
        "value": kvb / statistics.median(times) / 1e12, "unit": UNIT, "cores": info.get("threads_used", cores),
        "cores_asked": cores, "kind": "port", "seconds_per_call": statistics.median(times), "calls": len(times),
        "sample": f"{desc}; median of {len(times)} calls of the oracle's C restatement (OpenMP, "
                  f"{info.get('units', '?')} parallel units)"}
    return res


def _cpu_baseline_obj(res: dict) -> dict:
    main = res.get("reference", res["port"])
    cpu = {k: main[k] for k in ("value", "unit", "cores", "kind", "sample")}
    cpu["cores_asked"] = main["cores_asked"]
    if "reference" in res:
        cpu["port"] = {k: res["port"][k] for k in ("value", "cores", "kind")}
    else:
        cpu["note"] = "baseline/_ref holds no reference install; the oracle's C restatement stands in"
    return cpu


def run_reference_arm(args) -> None:
    rank, world, _ = _dist()
    if rank != 0:
        return
    res = cpu_measure(args.workload, steps=args.steps, warmup=args.warmup)
    main = res.get("reference", res["port"])
    v = main["value"]
    line = {
        "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": main["seconds_per_call"] * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": workload_config(args.workload, world, _seq_mode(args.workload, world, args.sharding), args.exchange),
        "cpu_baseline": _cpu_baseline_obj(res),
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def _parity_pick(lens) -> list[int]:
    live = [i for i, L in enumerate(lens) if L > 0]
    if not live:
        return [0]
    return sorted(set([live[0], max(live, key=lambda i: lens[i]), min(live, key=lambda i: lens[i])]
                      + [i for i, L in enumerate(lens) if L == 0][:1]))


def _oracle_own_heads(batch, pick):
    """The C oracle's output for sequences ``pick`` of this rank's batch (its own heads)."""
    from decodekernels_b200 import workloads
    from oracle import native

    q, kv = workloads.compact_sequences(batch, pick)
    kv = workloads.dequantize(kv, batch.config)  # e4m3 configs: the exact 16-bit values of the codes
    return native.dense_c(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, num_threads=_usable_cores())


def _errs(got, ref) -> tuple[bool, float, float]:
    import numpy as np

    err = np.abs(got - ref)
    ok = bool(np.isfinite(got).all() and err.max() <= MAX_ABS and err.mean() <= MEAN_ABS)
    return ok, float(err.max()), float(err.mean())


def _check_parity(batch, out) -> dict:
    """Sample sequences of this rank's output (its own heads) against the C oracle."""
    pick = _parity_pick(batch.lens)
    ok, mx, mean = _errs(out[pick].float().cpu().numpy(), _oracle_own_heads(batch, pick))
    return {"ok": ok, "sequences": pick, "max_abs": mx, "mean_abs": mean}


def _all_ok(ok: bool, world: int, dev) -> bool:
    """Every rank's verdict (a collective every rank makes, pass or fail)."""
    if world == 1:
        return ok
    import torch
    import torch.distributed as dist

    t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def _gather_parity_heads(batch, full_out, world, dev) -> dict:
    """Head sharding: every head of the gathered output on this rank -- the
    rank's own and those that arrived from its peers -- against the C oracle.
    Each rank computes the oracle for its own heads (it holds only their
    pages); an NCCL all-gather assembles the whole reference on every rank."""
    import torch
    import torch.distributed as dist

    pick = _parity_pick(batch.lens)
    ref = torch.from_numpy(_oracle_own_heads(batch, pick)).to(dev)
    parts = [torch.empty_like(ref) for _ in range(world)]
    dist.all_gather(parts, ref)
    ref_full = torch.cat(parts, dim=1).cpu().numpy()  # rank r's heads are [r * Hq/G, (r + 1) * Hq/G)
    ok, mx, mean = _errs(full_out[pick].float().cpu().numpy(), ref_full)
    return {"ok": ok, "sequences": pick, "heads": int(full_out.shape[1]), "max_abs": mx, "mean_abs": mean}


def _gather_parity_seq(batch, out, world, dev) -> dict:
    """Sequence sharding: the merged output on this rank against the oracle.
    Each rank computes the oracle's (o, lse) over its own blocks of the
    sample sequences; an NCCL all-gather and the oracle's log-sum-exp merge
    give the whole-sequence reference (exact: the token sets are disjoint)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from decodekernels_b200 import workloads
    from oracle import sharded_lse

    pick = _parity_pick(workloads.seq_lens(batch.config.name))
    q, kv = workloads.compact_sequences(batch, pick)
    kv = workloads.dequantize(kv, batch.config)
    o, lse = sharded_lse.attention_lse(q, kv.k_cache, kv.v_cache, kv.block_tables.numpy(), kv.seq_lens.numpy())
    o_t, l_t = torch.from_numpy(o).to(dev), torch.from_numpy(lse).to(dev)
    o_all, l_all = [torch.empty_like(o_t) for _ in range(world)], [torch.empty_like(l_t) for _ in range(world)]
    dist.all_gather(o_all, o_t)
    dist.all_gather(l_all, l_t)
    ref, _ = sharded_lse.merge_lse(np.stack([t.cpu().numpy() for t in o_all]),
                                   np.stack([t.cpu().numpy() for t in l_all]))
    ok, mx, mean = _errs(out[pick].float().cpu().numpy(), ref)
    return {"ok": ok, "sequences": pick, "heads": int(out.shape[1]), "max_abs": mx, "mean_abs": mean}


def _time_steps(step, steps, stream, flush_buf=None) -> float:
    """Device seconds of ``steps`` calls.  Without a flush the calls run back
    to back between one pair of CUDA events (as a serving loop issues them;
    per-call events between launches would stop a call's prologue from
    overlapping the previous call's tail).  With a flush, each call is
    bracketed by its own events and the flush stays outside them."""
    import torch

    if flush_buf is None:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(steps):
            step()
        e.record(stream)
        torch.cuda.synchronize()
        return s.elapsed_time(e) * 1e-3
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush_buf.zero_()
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    return sum(s.elapsed_time(e) for s, e in zip(starts, ends)) * 1e-3


_FLUSH = None


def _time_reference_method(fn, dev, warmup: int = 10, iters: int = 100) -> dict:
    """The reference benchmark's timing (benchmarks/bench_utils.py:33-52 of
    DecodeKernels: 10 warm-up calls, then per-call CUDA events around each of
    100 calls with a 256 MB buffer overwritten before each; median and
    10th / 90th percentiles)."""
    import torch

    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.int32, device=dev)
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    for i in range(iters):
        _FLUSH.zero_()
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize()
    us = sorted(s.elapsed_time(e) * 1e3 for s, e in zip(starts, ends))
    return {"median_us": statistics.median(us), "p10_us": us[int(0.1 * (len(us) - 1))],
            "p90_us": us[int(0.9 * (len(us) - 1))]}


def _vs_reference_kernel(batch, out, dev, ours_fn) -> dict:
    """The reference's CUDA kernel (its csrc/paged_attention.cuh built for
    sm_100a) on the same device tensors: its output against ours, and both
    timed the reference benchmark's way."""
    import numpy as np
    import torch

    from oracle import native

    if batch.config.kv_fp8:
        return {"reference_kernel": "none: the reference has no e4m3 KV path"}
    if not native.have_reference_kernel():
        return {"reference_kernel": "not built (oracle/_ref needs the reference source tree at build time)"}
    q, kv = batch.q, batch.kv
    n, hq, d = q.shape
    max_len = batch.max_seq_len
    rws = native.reference_workspace(n, hq, d, max_len, dev)
    rout = torch.empty_like(q)

    def ref_fn():
        native.reference_kernel(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, d**-0.5, max_len, rout, rws)

    ref_fn()
    torch.cuda.synchronize()
    diff = np.abs(rout.float().cpu().numpy() - out.float().cpu().numpy())
    ours = _time_reference_method(ours_fn, dev)
    ref = _time_reference_method(ref_fn, dev)
    del rws, rout
    return {"reference_kernel_us": _sig(ref["median_us"]), "ours_us_same_method": _sig(ours["median_us"]),
            "vs_reference_kernel": _sig(ref["median_us"] / ours["median_us"]),
            "outputs_max_abs_diff": _sig(float(diff.max()), 3),
            "method": "median of 100 calls, 256 MB L2 flush before each, 10 warm-up calls"}


def _flashinfer(batch, out, dev, ours_us: float) -> dict:
    """FlashInfer's batch decode (the baseline of DecodeKernels' own benchmark,
    benchmarks/bench_kernels.py:60-85) on the same batch: CUDA-core and
    tensor-core variants, each on contiguous NHD copies of the caches (its
    native layout; the copies are made before timing), checked against this
    library's output and timed the reference benchmark's way."""
    import itertools

    import numpy as np
    import torch

    try:
        import flashinfer
    except Exception as e:  # noqa: BLE001
        return {"error": f"flashinfer import failed: {e}"[:200]}
    if batch.config.kv_fp8 or min(batch.lens) <= 0:
        return {"error": "skipped: e4m3 caches or empty sequences"}
    q, kv = batch.q, batch.kv
    n, hq, d = q.shape
    hkv, bs = kv.k_cache.shape[2], kv.block_size
    blocks = [-(-L // bs) for L in batch.lens]
    indptr = torch.tensor([0] + list(itertools.accumulate(blocks)), dtype=torch.int32, device=dev)
    indices = torch.cat([kv.block_tables[i, :b] for i, b in enumerate(blocks)]).to(torch.int32)
    last = torch.tensor([(L - 1) % bs + 1 for L in batch.lens], dtype=torch.int32, device=dev)
    k_nhd, v_nhd = kv.k_cache.contiguous(), kv.v_cache.contiguous()
    ws = torch.zeros(128 * 1024 * 1024, dtype=torch.uint8, device=dev)
    res = {"version": getattr(flashinfer, "__version__", "?"), "ours_us_same_method": _sig(ours_us)}
    for tc in (False, True):
        key = "tensor_cores" if tc else "cuda_cores"
        try:
            w = flashinfer.BatchDecodeWithPagedKVCacheWrapper(ws, kv_layout="NHD", use_tensor_cores=tc)
            w.plan(indptr, indices, last, hq, hkv, d, bs, q_data_type=q.dtype, kv_data_type=q.dtype,
                   sm_scale=d**-0.5)

            def fn():
                return w.run(q, (k_nhd, v_nhd))

            o = fn()
            torch.cuda.synchronize()
            diff = float(np.abs(o.float().cpu().numpy() - out.float().cpu().numpy()).max())
            t = _time_reference_method(fn, dev)
            res[key] = {"us": _sig(t["median_us"]), "ours_speedup": _sig(t["median_us"] / ours_us),
                        "max_abs_diff_vs_ours": _sig(diff, 3)}
        except Exception as e:  # noqa: BLE001
            res[key] = {"error": f"{type(e).__name__}: {e}"[:300]}
    del k_nhd, v_nhd, ws
    return res


def _also(names, steps, warmup, dev, peaks, flashinfer: bool = False) -> dict:
    """Other workloads on this GPU: device-timed TB/s and roofline fraction
    (same method as the headline), a parity spot check, and the comparison
    with the reference's kernel."""
    import torch

    import decodekernels_b200 as dk
    from decodekernels_b200 import workloads

    res = {}
    stream = torch.cuda.current_stream(dev)
    for name in names:
        batch = workloads.make(name, dev)
        q, kv = batch.q, batch.kv
        n, hq, d = q.shape
        out = torch.empty_like(q)
        ws = dk.alloc_workspace(n, hq, d, batch.max_seq_len, dev, num_kv_heads=kv.k_cache.shape[2],
                                block_size=kv.block_size, merge_counters=True)
        sc = batch.config.kv_scale if batch.config.kv_fp8 else 1.0

        def step():
            dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens,
                                      max_seq_len=batch.max_seq_len, out=out, workspace=ws, k_scale=sc, v_scale=sc)

        step()
        torch.cuda.synchronize()
        parity = _check_parity(batch, out)
        flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.int32, device=dev) \
            if batch.kv_bytes() < FLUSH_BELOW else None
        for _ in range(warmup):
            step()
        t = _time_steps(step, steps, stream, flush) / steps
        entry = {"us_per_call": _sig(t * 1e6), "value": _sig(batch.kv_bytes() / t / 1e12),
                 "frac": _sig(batch.algorithmic_bytes() / t / 1e9 / peaks["hbm_gbs"]),
                 "l2_flush": flush is not None, "parity_ok": parity["ok"],
                 "parity_max_abs": _sig(parity["max_abs"], 3)}
        entry.update(_vs_reference_kernel(batch, out, dev, step))
        if flashinfer:
            ours_us = entry.get("ours_us_same_method") or _time_reference_method(step, dev)["median_us"]
            entry["flashinfer"] = _flashinfer(batch, out, dev, ours_us)
        res[name] = entry
        del batch, q, kv, out, ws, flush
        torch.cuda.empty_cache()
    return res


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

    seq_mode = _seq_mode(args.workload, world, args.sharding)
    config = workload_config(args.workload, world, seq_mode, args.exchange)
    if seq_mode:
        # Sequence sharding: every rank holds its striped blocks of every
        # sequence and the whole query; a step is the rank's partials, their
        # exchange and the log-sum-exp merge (full output on every rank).
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
    sc = batch.config.kv_scale if batch.config.kv_fp8 else 1.0
    plan = capi.plan(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, d**-0.5, max_len, out, ws,
                     k_scale=sc, v_scale=sc)
    dtype_str = "e4m3 KV, f16 mma" if batch.config.kv_fp8 else (
        "f16" if batch.config.dtype == torch.float16 else "bf16")

    if seq_mode:
        def step():
            seq_attn(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, max_seq_len=full_max, out=out,
                     workspace=ws, k_scale=sc, v_scale=sc)
    else:
        def step():
            dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, max_seq_len=max_len,
                                      out=out, workspace=ws, k_scale=sc, v_scale=sc)

    step()
    torch.cuda.synchronize()
    parity = _gather_parity_seq(batch, out, world, dev) if seq_mode else _check_parity(batch, out)
    if not _all_ok(parity["ok"], world, dev):
        if world > 1:
            torch.distributed.destroy_process_group()
        raise SystemExit(f"rank {rank}: parity check failed before timing: {parity}")

    # Inputs several times the 126 MB L2 (c2-c5) stream through it with no
    # reuse between steps; smaller ones (c1) get a 256 MB write between steps.
    flush = config["l2"].startswith("L2 flushed")
    flush_buf = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.int32, device=dev) if flush else None

    sampler = ClockSampler([local] if world == 1 else list(range(world))) if rank == 0 else None
    if sampler:
        sampler.start()

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        if flush:
            flush_buf.zero_()
        step()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    device_s = _time_steps(step, args.steps, stream, flush_buf)
    if world > 1:
        torch.distributed.barrier()
    t1 = time.perf_counter()
    if sampler:
        sampler.stop()

    # With N GPUs, also time the variant whose consumer needs every head on
    # every rank: decode + all-gather of the per-head outputs -- with
    # --exchange p2p the gather rides on the decode's output stores (peer
    # stores over NVLink, dk_paged_attention_decode_gather), with nccl an
    # all_gather_into_tensor follows the decode.  Every gathered head is
    # checked against the oracle before it is timed.
    gather_s = None
    gatherer = None
    gather_parity = parity if seq_mode else None
    if world > 1 and not seq_mode:
        from decodekernels_b200.sharded import ShardedPagedAttention

        gatherer = ShardedPagedAttention(batch.config.num_q_heads, batch.config.num_kv_heads, rank, world,
                                         exchange=args.exchange)
        full_out = torch.full((out.shape[0], batch.config.num_q_heads, out.shape[2]), float("nan"), dtype=out.dtype,
                              device=dev)

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
        gather_parity = _gather_parity_heads(batch, full_out, world, dev)
        own = torch.equal(full_out[:, rank * out.shape[1]:(rank + 1) * out.shape[1]], out)
        gather_parity["own_heads_equal_decode"] = own
        if not _all_ok(gather_parity["ok"] and own, world, dev):
            torch.distributed.destroy_process_group()
            raise SystemExit(f"rank {rank}: the gathered heads fail the oracle check: {gather_parity}")
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
                     k_scale=sc, v_scale=sc)
        else:
            dk.paged_attention_decode(qd, kv.k_cache, kv.v_cache, btd, sld, max_seq_len=max_len, out=outs[b],
                                      workspace=ws, k_scale=sc, v_scale=sc)

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
    if not _all_ok(torch.equal(e2e_out, dev_out), world, dev):
        diff = (e2e_out - dev_out).abs()
        if world > 1:
            torch.distributed.destroy_process_group()
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
    local_step = device_s / args.steps
    stats = torch.tensor([device_s, e2e_s, gather_s or 0.0, float(kv_local), float(alg_local)], dtype=torch.float64,
                         device=dev)
    gp = None
    if world > 1:
        import torch.distributed as dist

        tmax = stats[:3].clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        sums = stats[3:].clone()
        dist.all_reduce(sums, op=dist.ReduceOp.SUM)
        device_s, e2e_s, gather_s = tmax.tolist()
        kv_total, alg_total = sums.tolist()
        errs = torch.tensor([gather_parity["max_abs"], gather_parity["mean_abs"]], dtype=torch.float64, device=dev)
        per_rank = [torch.empty_like(errs) for _ in range(world)]
        dist.all_gather(per_rank, errs)
        gp = {"ok": True, "checked": ("the merged output of the sequence shards" if seq_mode else
                                      "every head of the gathered output"),
              "ranks": world, "sequences": gather_parity["sequences"], "heads": gather_parity["heads"],
              "vs": "CPU oracle (each rank's piece computed from its own pages, all-gathered over NCCL)",
              "max_abs_per_rank": [_sig(float(t[0]), 3) for t in per_rank],
              "mean_abs_per_rank": [_sig(float(t[1]), 3) for t in per_rank]}
    else:
        kv_total, alg_total = float(kv_local), float(alg_local)

    reference_kernel = None
    also = None
    if rank == 0 and world == 1 and not args.no_also:
        reference_kernel = _vs_reference_kernel(batch, out, dev, step)
        names = [w for w in args.also.split(",") if w and w != args.workload]
        if names:
            del ws, out, q, kv, batch, outs, d_stage, ins  # the headline batch is no longer needed
            torch.cuda.empty_cache()
            also = _also(names, max(args.steps, 100), args.warmup, dev, _peaks(), not args.no_flashinfer)

    if rank == 0:
        step_s = device_s / args.steps
        value = kv_total / step_s / 1e12
        peaks = _peaks()
        # roofline of this rank's calls: algorithmic bytes per call / mean call time
        achieved = alg_local / local_step / 1e9
        traffic = _profile_traffic(args.workload) if world == 1 else None
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_s * 1e3, "us_per_call": step_s * 1e6,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": dtype_str, "accumulate": "f32", "data": "synthetic", "impl": "ours",
            "config": config,
            "algorithmic_bytes_total": alg_total,
            "plan": plan, "parity": {k: parity[k] for k in ("sequences", "max_abs", "mean_abs")},
            "roofline": {
                "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                "peak_source": f"{peaks['source']} HBM copy bandwidth",
                "note": "achieved = algorithmic bytes per call / (CUDA-event time of the K back-to-back calls / K); "
                        "every kernel of the call counted",
            },
            "e2e": {"value": kv_total / (e2e_s / e_steps) / 1e12, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e_steps, "api": "decodekernels_b200.paged_attention_decode",
                    "copies": "pinned host buffers; each step's inputs (q, block tables, lengths in one staging "
                              "buffer) H2D and its output D2H on one copy stream per direction, double buffered, "
                              "overlapping the neighbouring steps' decode"},
            "gpu_launches": args.steps * (plan["launches"] + (1 if seq_mode else 0)),
            "exchange_errors": (seq_attn.p2p_errors() if seq_mode
                                else gatherer.p2p_errors() if gatherer is not None else None),
            "gather_parity": gp,
            "with_gather": None if not gather_s else {
                "us_per_call": gather_s / args.steps * 1e6, "value": kv_total / (gather_s / args.steps) / 1e12,
                "unit": UNIT, "note": "decode + all-gather of the per-head outputs to every rank ("
                + ("NCCL)" if args.exchange != "p2p" else
                   "one NVLink peer-memory kernel after the decode, dk_gather_heads)" if "f8" in args.workload else
                   "fused into the decode's output stores over NVLink peer memory, dk_paged_attention_decode_gather)")},
            "clocks": sampler.summary(t0, t1) if sampler else None,
            "wall_s_timed": t1 - t0,
        }
        if reference_kernel is not None:
            line["reference_kernel"] = reference_kernel
        if also is not None:
            line["also"] = also
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = _cpu_baseline_obj(cpu_measure(args.workload, seconds=args.cpu_seconds))
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
    ap.add_argument("--also", default="c2,c3,c4,c2f8,c3f8,c4f8",
                    help="N=1: other workloads timed after the headline (comma-separated; empty for none)")
    ap.add_argument("--no-also", action="store_true",
                    help="skip the reference-kernel comparison and the other workloads")
    ap.add_argument("--no-flashinfer", action="store_true",
                    help="N=1: skip FlashInfer's batch decode on the 16-bit workloads under --also")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
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
