#!/usr/bin/env python
"""Benchmark of the B200 GGUF weight-preparation path.

One step converts a whole model-shaped GGUF tensor set (default: the Llama-3-8B
Q4_K_M-shaped set, 291 tensors, 5.31 GB of GGUF bytes) into the reference's integer
layout (int8/int4 codes + f32 block scales).  With N GPUs (torchrun, one process per
GPU) the tensors are sharded by bytes across the ranks with no collective on the data
path; the model stays the same, so scaling is strong (fixed total work).

Printed (rank 0, one JSON line): whole-job GGUF GB/s with inputs resident in HBM
(`value`), seconds per model, the end-to-end number through the C ABI host-buffer call
(`gq_convert_host`, pinned host input -> pinned host output, copies inside the timed
region), the roofline of the dominant kernel, SM clocks sampled during the timed region,
and the CPU baseline (the numpy oracle on the host cores, rank 0 at N=1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--model llama3-8b] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "GGUF weight GB/s dequant+requant (frac. of HBM peak) and s/model at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--model", default="llama3-8b", choices=["llama3-8b", "qwen2.5-7b", "llama3-70b"])
    ap.add_argument("--out", default="codes", choices=["codes", "f32", "both"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-modalix", action="store_true",
                    help="skip the conversion fused with the Modalix layout (gq_convert_modalix)")
    ap.add_argument("--layers", type=int, default=0,
                    help="keep only the first L transformer layers (small cases for profiling)")
    ap.add_argument("--formats", default="", help="comma list of GGML formats to keep (profiling)")
    ap.add_argument("--tensor", default="",
                    help="FMT:ROWS:COLS: instead of a model set, --copies seeded copies of one tensor "
                         "(a BASELINE single-tensor config), all converted by one launch per step")
    ap.add_argument("--copies", type=int, default=8)
    ap.add_argument("--no-sustained", action="store_true", help="skip the >= 1 s steady-state timing")
    ap.add_argument("--sustained-seconds", type=float, default=1.5)
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the BASELINE config sub-records (C1 Q8_0, C2 Q4_0 / Q4_K, C4 Qwen2.5-7B set)")
    ap.add_argument("--no-70b", action="store_true", help="skip the Llama-3-70B set sub-record")
    return ap.parse_args()


def selected_specs(args):
    """The model's tensor list, optionally cut to the first --layers layers / --formats, or
    --copies copies of the single --tensor."""
    from llima_b200.synth import TensorSpec, model_specs
    if args.tensor:
        fmt, rows, cols = args.tensor.split(":")
        return [TensorSpec(f"{fmt}_{rows}x{cols}.{i}", fmt, int(rows), int(cols), 9000 + i)
                for i in range(args.copies)]
    specs = model_specs(args.model, args.seed)
    if args.layers:
        keep = []
        for s in specs:
            if s.name.startswith("blk."):
                if int(s.name.split(".")[1]) < args.layers:
                    keep.append(s)
        specs = keep
    if args.formats:
        fm = set(args.formats.split(","))
        specs = [s for s in specs if s.fmt in fm]
    return specs


# ---------------------------------------------------------------------------------------
# CPU side: the numpy oracle, timed on the host cores (spawned workers)
# ---------------------------------------------------------------------------------------

def _cpu_worker(model, seed, rank, sample_mb, seconds, passes, barrier, queue):
    import numpy as np  # noqa: F401
    sys.path.insert(0, str(ROOT))
    from llima_b200.synth import gen_tensor_bytes, model_specs
    from oracle import ggml_oracle as O

    # A slice of the model with its format mix: whole rows of every quantized format,
    # in proportion to the bytes each format holds in the model.
    specs = [s for s in model_specs(model, seed) if s.fmt != "F32"]
    by_fmt: dict[str, int] = {}
    for s in specs:
        by_fmt[s.fmt] = by_fmt.get(s.fmt, 0) + s.nbytes
    total = sum(by_fmt.values())
    sample = []
    for fmt, nb in sorted(by_fmt.items()):
        f = O.FORMATS[fmt]
        share = sample_mb * (1 << 20) * nb / total
        units = max(1, int(share // f.unit_bytes))
        n_values = units * f.unit_values
        raw = gen_tensor_bytes(fmt, n_values, seed * 7919 + rank * 31 + len(sample))
        sample.append((fmt, raw.tobytes(), n_values))
    nbytes = sum(len(r) for _, r, _ in sample)
    barrier.wait()
    t0 = time.time()
    done = 0
    n_pass = 0
    while True:
        for fmt, raw, n_values in sample:
            O.unpack_tensor(fmt, raw, (n_values // 256 if n_values % 256 == 0 else n_values // 32,
                                       256 if n_values % 256 == 0 else 32), log=False)
        done += nbytes
        n_pass += 1
        if (passes and n_pass >= passes) or (not passes and time.time() - t0 >= seconds):
            break
    queue.put((done, t0, time.time()))


def _cpu_step_worker(model, seed, rank, sample_mb, n_steps, barrier, queue):
    """One worker of the reference arm: n_steps synchronized passes over its sample."""
    sys.path.insert(0, str(ROOT))
    from llima_b200.synth import gen_tensor_bytes, model_specs
    from oracle import ggml_oracle as O
    specs = [s for s in model_specs(model, seed) if s.fmt != "F32"]
    by_fmt: dict[str, int] = {}
    for s in specs:
        by_fmt[s.fmt] = by_fmt.get(s.fmt, 0) + s.nbytes
    total = sum(by_fmt.values())
    sample = []
    for fmt, nb in sorted(by_fmt.items()):
        f = O.FORMATS[fmt]
        units = max(1, int(sample_mb * (1 << 20) * nb / total // f.unit_bytes))
        n_values = units * f.unit_values
        sample.append((fmt, gen_tensor_bytes(fmt, n_values, seed * 7919 + rank * 31 + len(sample)).tobytes(),
                       n_values))
    nbytes = sum(len(r) for _, r, _ in sample)
    times = []
    for _ in range(n_steps):
        barrier.wait()
        t0 = time.time()
        for fmt, raw, n_values in sample:
            O.unpack_tensor(fmt, raw, (n_values // 256 if n_values % 256 == 0 else n_values // 32,
                                       256 if n_values % 256 == 0 else 32), log=False)
        times.append((t0, time.time()))
    queue.put((nbytes, times))


def cpu_steps(model, seed, cores, sample_mb, n_steps):
    """Per-step (GGUF bytes, wall seconds) of `cores` workers converting their samples in
    lock step: a step's wall time is the last end minus the first start."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    barrier = ctx.Barrier(cores)
    queue = ctx.Queue()
    procs = [ctx.Process(target=_cpu_step_worker, args=(model, seed, r, sample_mb, n_steps, barrier, queue))
             for r in range(cores)]
    for p in procs:
        p.start()
    res = [queue.get() for _ in procs]
    for p in procs:
        p.join()
    total = sum(r[0] for r in res)
    out = []
    for i in range(n_steps):
        t0 = min(r[1][i][0] for r in res)
        t1 = max(r[1][i][1] for r in res)
        out.append((total, t1 - t0))
    return out


def cpu_throughput(model, seed, cores, sample_mb=8.0, seconds=8.0, passes=0):
    """GB/s of GGUF bytes converted by `cores` spawned processes running the oracle."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    barrier = ctx.Barrier(cores)
    queue = ctx.Queue()
    procs = [ctx.Process(target=_cpu_worker, args=(model, seed, r, sample_mb, seconds, passes, barrier, queue))
             for r in range(cores)]
    for p in procs:
        p.start()
    res = [queue.get() for _ in procs]
    for p in procs:
        p.join()
    total = sum(r[0] for r in res)
    wall = max(r[2] for r in res) - min(r[1] for r in res)
    return total / wall / 1e9, total, wall


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int]):
        self.gpus = set(gpus)
        self.proc = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        self.proc.wait()
        self.file.flush()
        self.file.seek(0)
        sm, mx, pw, reasons = [], [], [], set()
        capped = 0
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.file.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in self.gpus:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            try:
                pw.append(float(parts[3]))
            except ValueError:
                pass
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
                    capped += n == "sw_power_cap"
        os.unlink(self.file.name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons), "sw_power_cap_share": round(capped / len(sm), 3),
                "power_w_median": statistics.median(pw) if pw else None}


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


def traffic_per_byte(kernel: str):
    """DRAM bytes per algorithmic byte of `kernel`, from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return float(json.loads(p.read_text())[kernel]["dram_bytes_per_algorithmic_byte"])
    except (KeyError, ValueError, TypeError):
        return None


def workload_config(args, world) -> dict:
    from llima_b200.formats import output_layout
    specs = selected_specs(args)
    gguf = sum(s.nbytes for s in specs)
    out = 0
    for s in specs:
        lay = output_layout(s.fmt, s.n_values)
        if lay["codes"] == 0:
            out += lay["values"]
        else:
            out += (lay["codes"] + lay["scales"] if args.out in ("codes", "both") else 0) + \
                (lay["values"] if args.out in ("f32", "both") else 0)
    cut = ""
    if args.layers or args.formats:
        cut = f" (cut: layers={args.layers or 'all'}, formats={args.formats or 'all'})"
    workload = f"{args.model} GGUF tensor set, whole model per step{cut}"
    if args.tensor:
        workload = f"{args.copies} seeded copies of one {args.tensor} tensor, one launch per step"
    return {"workload": workload, "model": args.model if not args.tensor else args.tensor,
            "n_tensors": len(specs), "gguf_bytes": gguf, "out_bytes": out, "output": args.out,
            "parallelism": f"tensor-shard x{world}",
            "l2": "inputs larger than L2 (GGUF bytes >> 126 MB), no flush"}


def gguf_file_e2e(tensors, host_src, layers: int | None = None):
    """The host-to-host paths a user of the reference's loader takes, on a real GGUF file:
    the rank's tensors (all of them, or the embedding, the output head and the first
    `layers` layers) written with gguf-py's writer to a scratch file (page-cached; /dev/shm
    when it has room).  Returns two records, or (None, None) when there is no room:

    * from_gguf_file: convert_gguf_file, every quantized tensor in one host call (warmed up
      once, then timed once on a fresh reader);
    * dropin: GgufModel.load_weight's path, one load_tensor call per quantized tensor on a
      fresh GGUFReader (its memory map's pages are read inside the timed loop), each result
      dropped before the next call."""
    import shutil
    import numpy as np
    import gguf
    from llima_b200.gguf_conversion import GgufReaderProxy, convert_gguf_file, load_tensor
    keep = [(t, hs) for t, hs in zip(tensors, host_src)
            if layers is None or not t.name.startswith("blk.") or int(t.name.split(".")[1]) < layers]
    total = sum(hs.numel() for _, hs in keep)
    need = int(1.2 * total) + (1 << 30)
    d = "/dev/shm" if os.path.isdir("/dev/shm") and shutil.disk_usage("/dev/shm").free > need \
        else tempfile.gettempdir()
    if shutil.disk_usage(d).free < need:
        return None, None
    path = os.path.join(d, f"llima_b200_bench_{os.getpid()}.gguf")
    cut = "whole model" if layers is None else f"embedding, output and the first {layers} layers"
    try:
        w = gguf.GGUFWriter(path, "llama")
        heads = {t.name.split(".")[-2]: t.perm_heads for t, _ in keep if t.perm_heads}
        n_layers = 1 + max([int(t.name.split(".")[1]) for t, _ in keep if t.name.startswith("blk.")] or [0])
        w.add_block_count(n_layers)
        if "attn_q" in heads:
            w.add_head_count(heads["attn_q"])
            w.add_head_count_kv(heads.get("attn_k", heads["attn_q"]))
        for t, hs in keep:
            raw = hs.numpy()
            if t.fmt == "F32":
                w.add_tensor(t.name, raw.view(np.float32).reshape(t.rows) if t.cols == 1
                             else raw.view(np.float32).reshape(t.rows, t.cols))
            else:
                w.add_tensor(t.name, raw.reshape(t.rows, -1), raw_shape=(t.rows, raw.size // t.rows),
                             raw_dtype=getattr(gguf.GGMLQuantizationType, t.fmt))
        w.write_header_to_file()
        w.write_kv_data_to_file()
        w.write_tensors_to_file()
        w.close()
        del w
        res = convert_gguf_file(path)
        del res
        t0 = time.perf_counter()
        res = convert_gguf_file(path)
        dt = time.perf_counter() - t0
        n = len(res)
        del res
        whole = {"value": round(total / dt / 1e9, 3), "unit": "GB/s", "seconds": round(dt, 4), "gguf_bytes": total,
                 "tensors": n, "cut": cut,
                 "api": "convert_gguf_file (GGUFReader memory map, one gq_convert_host call)"}
        perm = {t.name: t.perm_heads for t, _ in keep}
        # GgufModel.load_weight's path: the proxy's load_tensor, one call per quantized
        # tensor in file order, each result dropped before the next call
        listing = [rt for rt in gguf.GGUFReader(path).tensors if rt.tensor_type.name not in ("F32", "F16", "BF16")]
        names = [rt.name for rt in listing]
        qbytes = sum(int(rt.n_bytes) for rt in listing)
        del listing
        proxy = GgufReaderProxy(path, perm_heads_of=lambda n: perm.get(n, 0))
        t0 = time.perf_counter()
        for n in names:
            s_, w_ = proxy.load_tensor(n, False, perm.get(n, 0))
            del s_, w_
        dt = time.perf_counter() - t0
        del proxy
        dropin = {"value": round(qbytes / dt / 1e9, 3), "unit": "GB/s", "s_per_model": round(dt, 4),
                  "gguf_bytes": qbytes, "tensors": len(names), "cut": cut,
                  "readahead_mb": int(os.environ.get("LLIMA_B200_READAHEAD_MB", "1024")),
                  "api": "GgufReaderProxy.load_tensor (GgufModel.load_weight's path), one call per quantized "
                         "tensor of a fresh GGUFReader in file order: memory-mapped file in, numpy arrays out"}
        # the same calls converting each tensor on its own (no read-ahead)
        reader = gguf.GGUFReader(path)
        quant = [rt for rt in reader.tensors if rt.tensor_type.name not in ("F32", "F16", "BF16")]
        t0 = time.perf_counter()
        for rt in quant:
            s_, w_ = load_tensor(rt, False, perm.get(rt.name, 0))
            del s_, w_
        dt1 = time.perf_counter() - t0
        del quant, reader
        dropin["one_tensor_per_call"] = {"value": round(qbytes / dt1 / 1e9, 3), "unit": "GB/s",
                                         "s_per_model": round(dt1, 4)}
        return whole, dropin
    finally:
        if os.path.exists(path):
            os.unlink(path)


class DeviceSet:
    """One rank's shard of a tensor set resident in HBM: the GGUF bytes of its pieces (byte-
    balanced over the ranks, no exchange), their outputs, and one DeviceBatch per GGML type
    (one launch each per step)."""
    ORDER = ["Q4_K", "Q5_K", "Q6_K", "Q8_0", "Q4_0", "F32"]

    def __init__(self, specs, model, rank, world, dev, out_mask, out_name):
        import torch
        from llima_b200.device import DeviceBatch, DeviceTensor, alloc_outputs
        from llima_b200.formats import FORMATS
        from llima_b200.shard import piece_cost, plan_shards
        from llima_b200.synth import gen_tensor_bytes_torch, head_count_for
        plan = plan_shards([(s.fmt, s.rows, s.cols, head_count_for(model, s.name) > 0) for s in specs],
                           world, out_name)
        by_index: dict[int, list] = {}
        for pc in plan[rank]:
            by_index.setdefault(pc.index, []).append(pc)
        self.tensors = []
        for idx, plist in by_index.items():
            sp = specs[idx]
            full = gen_tensor_bytes_torch(sp.fmt, sp.n_values, sp.seed, dev, sp.kind)
            f = FORMATS[sp.fmt]
            row_bytes = sp.cols // f.unit_values * f.unit_bytes
            for pc in plist:
                src = full[pc.row0 * row_bytes:pc.row1 * row_bytes].clone()
                heads = head_count_for(model, sp.name) if pc.rows == sp.rows else 0
                t = DeviceTensor(sp.fmt, pc.rows, sp.cols, src, heads, name=sp.name)
                self.tensors.append(alloc_outputs(t, out_mask))
            del full
        torch.cuda.synchronize()
        self.batches = {}
        for fmt in self.ORDER:
            ts = [t for t in self.tensors if t.fmt == fmt]
            if ts:
                self.batches[fmt] = DeviceBatch(ts, out_mask)
        self.algo = {fmt: sum(piece_cost(fmt, t.rows, t.cols, out_name) for t in b.tensors)
                     for fmt, b in self.batches.items()}
        self.gguf_bytes = sum(t.src_bytes for t in self.tensors)
        self.out_bytes = sum(t.out_bytes for t in self.tensors)
        self.launches_per_step = sum(-(-len(b.tensors) // 256) for b in self.batches.values())

    def step(self, stream, ev=None):
        import torch
        for fmt, b in self.batches.items():
            if ev is not None:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                b.run(stream, reset_diag=False)
                e1.record(stream)
                ev[fmt].append((e0, e1))
            else:
                b.run(stream, reset_diag=False)

    def reset_diag(self, stream):
        for b in self.batches.values():
            b.run(stream, reset_diag=True)

    def free(self):
        import torch
        self.tensors = []
        self.batches = {}
        torch.cuda.synchronize()
        torch.cuda.empty_cache()


def rank_max(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def rank_sum(xs: list, world: int, dev) -> list:
    if world == 1:
        return [float(x) for x in xs]
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(x) for x in xs], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return [float(v) for v in t.tolist()]


def rank_gather(x: float, world: int, dev) -> list:
    """x of every rank, in rank order."""
    if world == 1:
        return [float(x)]
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(o.item()) for o in out]


def timed_steps(ds: DeviceSet, steps: int, warmup: int, world: int, dev, sampler=None, per_format=True):
    """Whole steps of `ds` timed with CUDA events on the launching stream between barriers
    and synchronizes; returns the max-over-ranks ms per step, this rank's per-format kernel
    ms per launch, every rank's kernel time per step (work_ms) and the clock record."""
    import torch
    import torch.distributed as dist
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()
    for _ in range(warmup):
        ds.step(stream)
    torch.cuda.synchronize()
    barrier()
    if sampler:
        sampler.start()
        time.sleep(0.3)
    ev = {fmt: [] for fmt in ds.batches} if per_format else None
    torch.cuda.synchronize()
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        ds.step(stream, ev)
    t1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop() if sampler else None
    ms_step = rank_max(t0.elapsed_time(t1), world, dev) / steps
    per_fmt = {fmt: sum(a.elapsed_time(b) for a, b in lst) / len(lst) for fmt, lst in ev.items()} if ev else {}
    work = rank_gather(sum(per_fmt.values()), world, dev) if ev else None
    return ms_step, per_fmt, work, clocks


def work_record(work: list | None) -> dict | None:
    if not work:
        return None
    return {"per_rank": [round(w, 4) for w in work], "max": round(max(work), 4), "min": round(min(work), 4),
            "unit": "ms of kernel time per step (sum of the rank's per-format launch events)"}



def pcie_copy_peak(dev, world: int, nbytes: int = 512 << 20, reps: int = 3) -> dict:
    """Pinned host <-> device copy bandwidth of this box, the ceiling of the end-to-end figure:
    host-to-device alone, device-to-host alone and both at once on two streams (each
    direction's rate while the other runs), timed with CUDA events, every rank at the same
    time (a multi-GPU run shares the host's memory and I/O path); GB/s summed over ranks."""
    import torch
    import torch.distributed as dist
    try:
        hs = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
        hd = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
        ds_ = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        dd = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        ok = 1.0
    except (RuntimeError, MemoryError):
        hs = hd = ds_ = dd = None
        ok = 0.0
    if world > 1:
        # every rank measures or none does (the measurement's barriers and sums are collective)
        t = torch.tensor([ok], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        ok = float(t.item())
    if ok < 1.0:
        return {"unavailable": "no room for the pinned copy-test buffers on every rank"}
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def run(h2d: bool, d2h: bool) -> tuple[float, float]:
        ev = {k: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for k in ("u", "d")}
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        for key, on, st, fn in (("u", h2d, up, lambda: ds_.copy_(hs, non_blocking=True)),
                                ("d", d2h, down, lambda: hd.copy_(dd, non_blocking=True))):
            if not on:
                continue
            with torch.cuda.stream(st):
                ev[key][0].record(st)
                for _ in range(reps):
                    fn()
                ev[key][1].record(st)
        torch.cuda.synchronize(dev)
        rate = lambda k: nbytes * reps / (ev[k][0].elapsed_time(ev[k][1]) / 1e3) / 1e9
        return (rate("u") if h2d else 0.0), (rate("d") if d2h else 0.0)

    run(True, True)   # warm-up
    h2d_alone, _ = run(True, False)
    _, d2h_alone = run(False, True)
    h2d_both, d2h_both = run(True, True)
    tot = rank_sum([h2d_alone, d2h_alone, h2d_both, d2h_both], world, dev)
    del hs, hd, ds_, dd
    return {"h2d_gbs": round(tot[0], 2), "d2h_gbs": round(tot[1], 2), "h2d_gbs_bidir": round(tot[2], 2),
            "d2h_gbs_bidir": round(tot[3], 2), "bytes_per_copy": nbytes, "copies": reps, "ranks": world}


def single_tensor_rate(fmt: str, rows: int, cols: int, dev, world: int, peak: float) -> dict:
    """One tensor per launch, as BASELINE's single-tensor configs give it.  Copies of the
    tensor (different seeds) rotate so that consecutive launches read more than L2 holds;
    one launch per copy is captured in a CUDA graph (a host call per launch would take
    longer than the kernel) and the graph is replayed, timed with CUDA events.  With N
    ranks every rank converts its own copies (replicas); the slowest rank is reported."""
    import torch
    import torch.distributed as dist
    from llima_b200 import _native as N
    from llima_b200.device import DeviceBatch, DeviceTensor, alloc_outputs
    from llima_b200.formats import FORMATS
    from llima_b200.shard import piece_cost
    from llima_b200.synth import gen_tensor_bytes_torch
    cost = piece_cost(fmt, rows, cols, "codes")
    n_copies = max(2, -(-3 * (126 << 20) // cost))
    copies = []
    for i in range(n_copies):
        src = gen_tensor_bytes_torch(fmt, rows * cols, 7000 + i, dev)
        copies.append(DeviceBatch([alloc_outputs(DeviceTensor(fmt, rows, cols, src), N.OUT_CODES)], N.OUT_CODES))
    stream = torch.cuda.current_stream()
    for b in copies:
        b.run(stream, reset_diag=True)
    for _ in range(3):
        for b in copies:
            b.run(stream, reset_diag=False)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for b in copies:
            b.run(reset_diag=False)
    g.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    reps = max(5, -(-2000 // n_copies))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = rank_max(e0.elapsed_time(e1), world, dev) / (reps * n_copies)
    del g
    f = FORMATS[fmt]
    gguf = rows * cols // f.unit_values * f.unit_bytes
    out = {"shape": [rows, cols], "format": fmt, "ms_per_launch": round(ms, 5),
           "value": round(gguf / (ms / 1e3) / 1e9, 1), "unit": "GB/s of GGUF",
           "hbm_frac": round(cost / (ms / 1e3) / 1e9 / peak, 4), "algorithmic_bytes": cost,
           "kernel": f"gq_convert_kernel<{fmt}>", "launches_timed": reps * n_copies,
           "copies": n_copies, "l2": "rotating copies, more than 3x L2 between reuses"}
    del copies
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from llima_b200 import _native as N
    from llima_b200.formats import FORMATS
    from llima_b200.shard import piece_cost

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    out_mask = {"codes": N.OUT_CODES, "f32": N.OUT_F32, "both": N.OUT_CODES | N.OUT_F32}[args.out]
    N.lib()   # fail loudly before any work if the library is missing

    specs = selected_specs(args)
    ds = DeviceSet(specs, args.model, rank, world, dev, out_mask, args.out)
    tensors = ds.tensors
    batches = ds.batches
    algo = ds.algo
    gguf_bytes = ds.gguf_bytes
    out_bytes = ds.out_bytes
    launches_per_step = ds.launches_per_step
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()

    ds.reset_diag(stream)
    sampler = ClockSampler([local_rank] if world == 1 else list(range(world))) if rank == 0 else None
    ms_step, per_fmt_ms, work, clocks = timed_steps(ds, args.steps, args.warmup, world, dev, sampler)

    # ---- the same step held for >= --sustained-seconds: the board's power cap engages
    # after a fraction of a second, so this is the rate a long conversion job runs at
    sustained = None
    if not args.no_sustained:
        n_sus = max(args.steps, int(args.sustained_seconds * 1e3 / max(ms_step, 1e-3)) + 1)
        sam = ClockSampler([local_rank] if world == 1 else list(range(world))) if rank == 0 else None
        ms_sus, _, _, clk_sus = timed_steps(ds, n_sus, 3, world, dev, sam, per_format=False)
        peak_, _ = measured_peak()
        tot_s = rank_sum([gguf_bytes, out_bytes], world, dev)
        sustained = {"value": round(tot_s[0] / (ms_sus / 1e3) / 1e9, 2), "unit": "GB/s", "steps": n_sus,
                     "seconds": round(n_sus * ms_sus / 1e3, 3), "ms_per_step": round(ms_sus, 4),
                     "hbm_frac_whole_step": round((tot_s[0] + tot_s[1]) / (ms_sus / 1e3) / 1e9 / (peak_ * world), 4),
                     "clocks": clk_sus}

    # correctness guard on the timed buffers: the diagnostics of the asymmetric formats
    # must have been written (rounding error of random data is > 0)
    diag_ok = True
    for fmt in ("Q4_K", "Q5_K"):
        if fmt in batches and out_mask & N.OUT_CODES:
            diag_ok &= bool((batches[fmt].diags[:, 0] != 0).any().item())

    # ---- the conversion fused with the Modalix weight layout: every quantized tensor of
    # this rank in one gq_convert_modalix_batch call (one launch per GGML type), against the
    # two passes it replaces (the conversion above plus gq_modalix_layout on its results,
    # one launch per tensor, captured in a CUDA graph)
    modalix = None
    if not args.no_modalix and out_mask == N.OUT_CODES:
        import ctypes
        keep, lrecs, mbytes, malgo = [], [], 0, 0
        quant = [t for t in tensors if FORMATS[t.fmt].block_values]
        mrecs = (N.Tensor * max(1, len(quant)))()
        for i, t in enumerate(quant):
            f = FORMATS[t.fmt]
            oc = torch.empty((t.cols, t.rows), dtype=torch.int8, device=dev)
            os_ = torch.empty((t.cols // f.block_values, t.rows), dtype=torch.float32, device=dev)
            r = N.Tensor()
            r.type, r.perm_heads, r.rows, r.cols = f.type_id, t.perm_heads, t.rows, t.cols
            r.src, r.src_bytes, r.codes, r.scales = t.src.data_ptr(), t.src.numel(), oc.data_ptr(), os_.data_ptr()
            mrecs[i] = r
            keep.append((oc, os_))
            lrecs.append((t, oc, os_, f.block_values))
            mbytes += t.src_bytes
            malgo += piece_cost(t.fmt, t.rows, t.cols, "codes")
        n_types = len({t.fmt for t in quant})

        def mstep():
            sid = torch.cuda.current_stream().cuda_stream
            N.check(N.lib().gq_convert_modalix_batch(mrecs, None, len(quant), sid), "gq_convert_modalix_batch")

        # launches go to the current stream (the capture stream while a graph is recorded)
        def lstep():
            sid = torch.cuda.current_stream().cuda_stream
            for t, oc, os_, blk in lrecs:
                N.check(N.lib().gq_modalix_layout(t.codes.data_ptr(), t.scales.data_ptr(), t.rows, t.cols, blk, t.rows,
                                                  oc.data_ptr(), os_.data_ptr(), sid), "gq_modalix_layout")

        def events_ms(fn, n, graph=False):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            g = None
            if graph:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    fn()
                run = g.replay
            else:
                run = fn
            run()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(n):
                run()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / n
            del g
            return ms

        if quant:
            barrier()
            m_ms = events_ms(mstep, 20)
            l_ms = events_ms(lstep, 20, graph=True)
            agg = torch.tensor([m_ms, l_ms], dtype=torch.float64, device=dev)
            tot = torch.tensor([float(mbytes), float(malgo)], dtype=torch.float64, device=dev)
            if world > 1:
                dist.all_reduce(agg, op=dist.ReduceOp.MAX)
                dist.all_reduce(tot, op=dist.ReduceOp.SUM)
            m_ms, l_ms = float(agg[0].item()), float(agg[1].item())
            peak_, _ = measured_peak()
            modalix = {"value": round(float(tot[0].item()) / (m_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                       "ms_per_model": round(m_ms, 4),
                       "hbm_frac": round(float(tot[1].item()) / (m_ms / 1e3) / 1e9 / (peak_ * world), 4),
                       "two_pass_ms_per_model": round(ms_step + l_ms, 4), "layout_pass_ms": round(l_ms, 4),
                       "launches_per_step": n_types, "api": "gq_convert_modalix_batch (one launch per GGML type)"}
        del mrecs, lrecs, keep

    # ---- token-embedding rows for the runtime (gq_embedding_rows: force_float dequantize,
    # x embed_scale, bf16 round, per-row int8 with a bf16 scale), on this rank's piece of
    # token_embd; traffic = GGUF bytes read + int8 codes + bf16 row scales written
    embedding = None
    if not args.no_modalix and out_mask == N.OUT_CODES:
        emb = [t for t in tensors if t.name == "token_embd.weight"]
        if emb:
            t = emb[0]
            f = FORMATS[t.fmt]
            codes_e = torch.empty((t.rows, t.cols), dtype=torch.int8, device=dev)
            scales_e = torch.empty((t.rows, 1), dtype=torch.uint16, device=dev)

            def estep():
                N.check(N.lib().gq_embedding_rows(f.type_id, t.src.data_ptr(), t.src.numel(), t.rows, t.cols, 1.0, 1,
                                                  codes_e.data_ptr(), scales_e.data_ptr(), None,
                                                  torch.cuda.current_stream().cuda_stream), "gq_embedding_rows")

            for _ in range(3):
                estep()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(20):
                estep()
            e1.record()
            torch.cuda.synchronize()
            e_ms = e0.elapsed_time(e1) / 20
            peak_, _ = measured_peak()
            moved = t.src_bytes + t.rows * t.cols + 2 * t.rows
            embedding = {"value": round(t.src_bytes / (e_ms / 1e3) / 1e9, 2), "unit": "GB/s", "ms": round(e_ms, 4),
                         "rows": t.rows, "cols": t.cols, "format": t.fmt,
                         "hbm_frac": round(moved / (e_ms / 1e3) / 1e9 / peak_, 4), "rank": rank,
                         "api": "gq_embedding_rows on this rank's token_embd rows (quantize=1)"}
            del codes_e, scales_e

    # ---- end to end through the C ABI host-buffer call (pinned host memory)
    e2e = None
    if not args.no_e2e and args.e2e_steps > 0:
        import ctypes
        host_src = []
        host_out = []
        recs = (N.Tensor * len(tensors))()
        for i, t in enumerate(tensors):
            hs = torch.empty(t.src.numel(), dtype=torch.uint8, pin_memory=True)
            hs.copy_(t.src)
            host_src.append(hs)
            r = N.Tensor()
            r.type = FORMATS[t.fmt].type_id
            r.perm_heads = t.perm_heads
            r.rows, r.cols = t.rows, t.cols
            r.src, r.src_bytes = hs.data_ptr(), hs.numel()
            outs = {}
            for name in ("codes", "scales", "values"):
                dt = getattr(t, name)
                if dt is not None:
                    ht = torch.empty(dt.shape, dtype=dt.dtype, pin_memory=True)
                    outs[name] = ht
                    setattr(r, name, ht.data_ptr())
            host_out.append(outs)
            recs[i] = r
        diags = (N.Diag * len(tensors))()
        sess = ctypes.c_void_p()
        N.check(N.lib().gq_session_create(local_rank, 1 << 30, ctypes.byref(sess)), "gq_session_create")
        N.check(N.lib().gq_convert_host(sess, recs, len(tensors), out_mask, diags), "gq_convert_host")  # warm-up
        barrier()
        times = []
        for _ in range(args.e2e_steps):
            barrier()
            t0 = time.perf_counter()
            N.check(N.lib().gq_convert_host(sess, recs, len(tensors), out_mask, diags), "gq_convert_host")
            times.append(time.perf_counter() - t0)
        barrier()
        e2e_s = sum(times) / len(times)
        if world > 1:
            t = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t.item())
        # the host results must equal the device-resident results
        same = True
        for t, outs in zip(tensors, host_out):
            for name, ht in outs.items():
                same &= bool(torch.equal(ht.to(dev, non_blocking=False).view(torch.uint8),
                                         getattr(t, name).view(torch.uint8)))
        N.lib().gq_session_destroy(sess)

        # The drop-in call the reference's GgufModel.load_weight makes, one tensor at a
        # time: pageable numpy input (as a memory-mapped GGUF file gives it) and freshly
        # allocated numpy results, through gguf_conversion.convert_host.  Float tensors
        # are passed through on the host by that API and are left out here.
        from llima_b200.gguf_conversion import convert_host as dropin
        quant = [(t, hs.numpy().copy()) for t, hs in zip(tensors, host_src) if FORMATS[t.fmt].block_values]
        if quant:
            t0_, r0_ = quant[0]
            dropin(t0_.fmt, r0_, t0_.rows, t0_.cols, False, t0_.perm_heads)   # session set-up
        barrier()
        t0 = time.perf_counter()
        for t, raw in quant:
            dropin(t.fmt, raw, t.rows, t.cols, False, t.perm_heads)
        dropin_s = time.perf_counter() - t0
        barrier()
        dropin_bytes = float(sum(r.size for _, r in quant))
        del quant
        # from a GGUF file on one GPU (ranks of a multi-GPU run would each need their own)
        file_e2e, file_dropin = gguf_file_e2e(tensors, host_src) if world == 1 else (None, None)
        h2d = sum(h.numel() for h in host_src)
        d2h = sum(ht.numel() * ht.element_size() for outs in host_out for ht in outs.values())
        agg = torch.tensor([float(gguf_bytes), float(h2d), float(d2h), 1.0 if same else 0.0, dropin_bytes],
                           dtype=torch.float64, device=dev)
        tmax = torch.tensor([dropin_s], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(agg, op=dist.ReduceOp.SUM)
            dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        # the copy engines' ceiling: the model's bytes in each direction at the rates both
        # directions reach together on this box
        pcie = pcie_copy_peak(dev, world)
        if "unavailable" not in pcie:
            bound_s = max(float(agg[1].item()) / (pcie["h2d_gbs_bidir"] * 1e9),
                          float(agg[2].item()) / (pcie["d2h_gbs_bidir"] * 1e9))
            pcie["bound_s_per_model"] = round(bound_s, 4)
            pcie["frac"] = round(bound_s / e2e_s, 4)
        e2e = {"value": float(agg[0].item()) / e2e_s / 1e9, "unit": "GB/s", "s_per_model": e2e_s,
               "pcie_roofline": pcie,
               "h2d_bytes_per_step": int(agg[1].item()), "d2h_bytes_per_step": int(agg[2].item()),
               "matches_device": bool(agg[3].item() == world), "api": "gq_convert_host (pinned host buffers)",
               "dropin_pageable": file_dropin,
               "dropin_numpy_copies": {"value": round(float(agg[4].item()) / float(tmax.item()) / 1e9, 3),
                                       "unit": "GB/s", "s_per_model": round(float(tmax.item()), 4),
                                       "api": "gguf_conversion.convert_host, one call per tensor, pageable numpy "
                                              "arrays in (not a memory map: bounced), numpy arrays out"},
               "from_gguf_file": file_e2e}
        del host_src, host_out

    # ---- the other BASELINE workloads, each after the previous one's memory is freed
    del tensors, batches
    ds.free()
    full_set = not (args.layers or args.formats or args.tensor) and out_mask == N.OUT_CODES
    peak_, _ = measured_peak()
    configs = None
    if not args.no_configs and out_mask == N.OUT_CODES:
        from llima_b200.synth import model_specs
        configs = {}
        for key, fmt, rows, cols in (("C1_Q8_0_4096x4096", "Q8_0", 4096, 4096),
                                     ("C2_Q4_0_11008x4096", "Q4_0", 11008, 4096),
                                     ("C2_Q4_K_11008x4096", "Q4_K", 11008, 4096)):
            configs[key] = single_tensor_rate(fmt, rows, cols, dev, world, peak_)
        if args.model != "qwen2.5-7b":
            qs = DeviceSet(model_specs("qwen2.5-7b", args.seed), "qwen2.5-7b", rank, world, dev, out_mask, "codes")
            qs.reset_diag(stream)
            ms_q, per_q, work_q, _ = timed_steps(qs, max(5, min(args.steps, 20)), 3, world, dev)
            tot_q = rank_sum([qs.gguf_bytes, qs.out_bytes], world, dev)
            configs["C4_qwen2.5-7b_set"] = {
                "value": round(tot_q[0] / (ms_q / 1e3) / 1e9, 2), "unit": "GB/s of GGUF",
                "ms_per_model": round(ms_q, 4),
                "hbm_frac": round((tot_q[0] + tot_q[1]) / (ms_q / 1e3) / 1e9 / (peak_ * world), 4),
                "gguf_bytes": int(tot_q[0]), "out_bytes": int(tot_q[1]), "work_ms": work_record(work_q),
                "per_format_GBps": {k: round(qs.algo[k] / (v / 1e3) / 1e9, 1) for k, v in per_q.items()},
                "per_format_frac": {k: round(qs.algo[k] / (v / 1e3) / 1e9 / peak_, 4) for k, v in per_q.items()}}
            qs.free()
    llama3_70b = None
    if not args.no_70b and full_set and args.model != "llama3-70b":
        from llima_b200.synth import model_specs
        ds70 = DeviceSet(model_specs("llama3-70b", args.seed), "llama3-70b", rank, world, dev, out_mask, "codes")
        ds70.reset_diag(stream)
        sam70 = ClockSampler([local_rank] if world == 1 else list(range(world))) if rank == 0 else None
        n70 = max(3, min(args.steps, 10))
        ms70, per70, work70, clk70 = timed_steps(ds70, n70, 2, world, dev, sam70)
        tot70 = rank_sum([ds70.gguf_bytes, ds70.out_bytes], world, dev)
        llama3_70b = {
            "s_per_model": round(ms70 / 1e3, 6), "value": round(tot70[0] / (ms70 / 1e3) / 1e9, 2),
            "unit": "GB/s of GGUF", "n_gpus": world, "steps": n70,
            "hbm_frac": round((tot70[0] + tot70[1]) / (ms70 / 1e3) / 1e9 / (peak_ * world), 4),
            "gguf_bytes": int(tot70[0]), "out_bytes": int(tot70[1]), "work_ms": work_record(work70),
            "per_format_GBps_rank0": {k: round(ds70.algo[k] / (v / 1e3) / 1e9, 1) for k, v in per70.items()},
            "clocks": clk70, "sharding": "tensors and row ranges byte-balanced over the ranks, no collective"}
        ds70.free()

    tot = torch.tensor([float(gguf_bytes), float(out_bytes), 1.0 if diag_ok else 0.0], dtype=torch.float64,
                       device=dev)
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
    all_gguf, all_out = float(tot[0].item()), float(tot[1].item())
    if rank != 0:
        return None

    peak, peak_kind = measured_peak()
    dom = max(per_fmt_ms, key=lambda f: per_fmt_ms[f])
    achieved = algo[dom] / (per_fmt_ms[dom] / 1e3) / 1e9
    tpb = traffic_per_byte(f"{dom.lower()}_convert")
    roofline = {"bound": "hbm", "kernel": f"gq_convert_kernel<{dom}>", "achieved": round(achieved, 1),
                "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "traffic": None if tpb is None else int(tpb * algo[dom]),
                "algorithmic_bytes_per_launch": algo[dom],
                "per_format_ms": {k: round(v, 4) for k, v in per_fmt_ms.items()},
                "per_format_GBps": {k: round(algo[k] / (v / 1e3) / 1e9, 1) for k, v in per_fmt_ms.items()}}
    value = all_gguf / (ms_step / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "s_per_model": round(ms_step / 1e3, 6),
        "hbm_frac_whole_step": round((all_gguf + all_out) / (ms_step / 1e3) / 1e9 / (peak * world), 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8->int8 (f32 requant)",
        "data": "synthetic (seeded, BASELINE distributions)",
        "config": workload_config(args, world),
        "roofline": roofline, "gpu_launches": launches_per_step * args.steps, "diag_written": bool(tot[2].item() == world),
        "work_ms": work_record(work), "sustained": sustained,
        "e2e": e2e, "clocks": clocks, "modalix_fused": modalix, "embedding_rows": embedding,
        "configs": configs, "llama3_70b": llama3_70b,
    }
    return line


def main():
    args = parse_args()
    # stdout carries exactly one JSON line: everything else any library writes to file
    # descriptor 1 (NCCL's version banner, for one) goes to stderr, and the result line is
    # written to the original stdout
    json_fd = os.dup(1)
    sys.stdout.flush()
    os.dup2(2, 1)

    def emit(line: dict) -> None:
        os.write(json_fd, (json.dumps(line) + "\n").encode())
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and world != 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)

    if args.impl == "reference":
        if rank != 0:
            return 0
        cores = host_cores()
        steps = cpu_steps(args.model, args.seed, cores, 4.0, args.warmup + args.steps)[args.warmup:]
        vals = [(total / wall / 1e9, total, wall) for total, wall in steps]
        value = sum(v[1] for v in vals) / sum(v[2] for v in vals) / 1e9
        sample = (f"per step: {cores} spawned workers, each converting a 4 MB slice of the {args.model} "
                  f"format mix (numpy oracle), steps synchronized by a barrier")
        line = {"metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(statistics.median(v[2] for v in vals) * 1e3, 2),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "u8->int8 (f32 requant)", "data": "synthetic (seeded, BASELINE distributions)",
                "config": workload_config(args, args.gpus),
                "impl": "reference",
                "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                                 "sample": sample},
                "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        emit(line)
        return 0

    import torch
    import torch.distributed as dist
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local_rank))
    try:
        cpu = None
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            # before any CUDA work: spawned workers, bounded by --cpu-seconds
            cores = host_cores()
            gbs, total, wall = cpu_throughput(args.model, args.seed, cores, sample_mb=8.0,
                                              seconds=args.cpu_seconds)
            # and one process alone, as the reference runs without its process pool
            gbs1, total1, wall1 = cpu_throughput(args.model, args.seed, 1, sample_mb=8.0,
                                                 seconds=max(2.0, args.cpu_seconds / 2))
            cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                   "sample": f"{cores} spawned workers, each an 8 MB slice of the {args.model} format mix "
                             f"converted repeatedly for {args.cpu_seconds:.0f} s ({total / 1e9:.2f} GB in {wall:.1f} s)",
                   "value_1_process": round(gbs1, 4),
                   "sample_1_process": f"1 spawned worker, the same 8 MB slice, {total1 / 1e9:.2f} GB in {wall1:.1f} s"}
        line = run_ours(args, rank, world, local_rank)
        if rank == 0 and line is not None:
            line["cpu_baseline"] = cpu
            emit(line)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
