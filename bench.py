#!/usr/bin/env python
"""SOAP atom-environments/s on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl ours|reference]

A step is one pass of the SOAP hot path (neighbour search, expansion, power
spectrum) over one batch of synthetic structures with the shape of the chosen
benchmark config (default: config 2, 1024 periodic 14 A cells x 128 atoms,
n_max 8, l_max 6, float32 output).  Multi-GPU runs are weak-scaled: each rank
owns its own seeded batch of that size (structures shard with no exchange).

* ``value``: device-resident throughput -- inputs already in HBM, output rows
  written to HBM, CUDA events on the launching stream around each step, L2
  flushed (256 MiB write) between steps outside the events; max over ranks.
* ``e2e``: the same metric through the public host API (``Soap.compute``):
  pinned host inputs uploaded and every output row copied back to pinned host
  memory inside the timed region.
* ``roofline``: the centre kernel (the dominant launch) against the measured
  HBM copy bandwidth (compulsory bytes), plus ``roofline_fp64`` against the
  measured fp64 FMA rate, the pipe that actually binds it.
* ``cpu_baseline``: the reference's own C++/OpenMP CPU SOAP (compiled from its
  sources into oracle/_ref) on a bounded sample, all host threads.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "SOAP atom-environments/sec"
UNIT = "atom-env/s"
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--config", type=int, default=2)
    p.add_argument("--structures", type=int, default=None, help="structures per rank (default: the config's)")
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--local", default=None, choices=("SphericalExpansion", "SoapRadialSpectrum", "SoapPowerSpectrum"),
                   help="time a local spherical spectrum (reference defaults) instead of SOAP; one GPU")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def rank_seed(config: int, rank: int) -> int:
    """Each rank owns its own seeded batch (weak scaling, no exchange)."""
    from mdescriptor_b200 import workloads

    return workloads.SEED_BASE + config + 1000 * rank


class Ranks:
    """One process per GPU, launched by torchrun (RANK/WORLD_SIZE/LOCAL_RANK).

    The only collectives are a barrier around the timed regions and the
    max / sum reductions of the per-rank timings and unit counts -- the SOAP
    path itself shards by structure with no exchange.  ``backend`` is "nccl"
    on GPUs and "gloo" for the CPU tests of this logic.
    """

    def __init__(self, backend: str = "nccl", device=None, timeout_s: float = 120.0):
        self.rank, self.world, self.local = dist_env()
        self.device = device
        self.group = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            kwargs = {"device_id": device} if backend == "nccl" else {}
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kwargs)
            self.group = dist

    def barrier(self):
        if self.group is not None:
            self.group.barrier()

    def _reduce(self, x: float, op) -> float:
        if self.group is None:
            return float(x)
        import torch

        t = torch.tensor([float(x)], dtype=torch.float64, device=self.device)
        self.group.all_reduce(t, op=op)
        return float(t.item())

    def max(self, x: float) -> float:
        return self._reduce(x, None if self.group is None else self.group.ReduceOp.MAX)

    def sum(self, x: float) -> float:
        return self._reduce(x, None if self.group is None else self.group.ReduceOp.SUM)

    def close(self):
        if self.group is not None:
            self.group.destroy_process_group()
            self.group = None


def job_throughput(units_all_ranks: float, steps: int, max_ms: float) -> float:
    """Whole-job units/s: every rank's units over the slowest rank's time."""
    return units_all_ranks * steps / (max_ms * 1e-3)


def config_record(args, cfg, structures, atoms, world, parallelism=None):
    return {
        "workload": f"{cfg.name} (BASELINE config {args.config})",
        "structures_per_rank": structures,
        "atoms_per_rank": atoms,
        "species": list(cfg.species),
        "r_cut": cfg.r_cut,
        "n_max": cfg.n_max,
        "l_max": cfg.l_max,
        "sigma": cfg.sigma,
        "average": cfg.average,
        "output_dtype": cfg.dtype,
        "parallelism": parallelism or f"structure-sharded x{world} (no collective)",
        "l2": "flushed between steps (256 MiB device write, outside the timed events)",
    }


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback (profiling recipe: 6.65 TB/s)"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons every 200 ms, timestamped on arrival.

    Started before the warm-up (nvidia-smi needs a moment to print its first
    sample); only samples that arrive inside a window marked with
    ``begin()``/``end()`` -- the timed regions -- enter the summary.
    """

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.samples: list[tuple[float, str]] = []
        self.windows: list[list[float]] = []
        self.thread = None
        self.first = threading.Event()

    def start(self, wait_s: float = 5.0):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        self.first.wait(wait_s)

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.monotonic(), line.strip()))
            self.first.set()

    def begin(self):
        self.windows.append([time.monotonic(), float("inf")])

    def end(self):
        if self.windows:
            self.windows[-1][1] = time.monotonic()

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        return summarize_clocks(self.samples, self.windows, self.NAMES)


def summarize_clocks(samples, windows, names=ClockSampler.NAMES):
    """Median SM clock, max clock and active reasons over samples inside the windows."""
    sm, sm_max, power, reasons = [], [], [], set()
    for t, line in samples:
        if not any(a <= t <= b for a, b in windows):
            continue
        parts = [x.strip() for x in line.split(",")]
        if len(parts) < 7:
            continue
        try:
            sm.append(float(parts[0]))
            sm_max.append(float(parts[1]))
        except ValueError:
            continue
        try:
            power.append(float(parts[2]))
        except ValueError:
            pass
        for name, flag in zip(names, parts[3:7]):
            if flag.lower() == "active":
                reasons.add(name)
    if not sm:
        return None
    return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(sm_max), "reasons": sorted(reasons),
            "samples": len(sm), "power_w_max": max(power) if power else None}


def algorithmic_flops_per_atom(cfg, edges_per_atom):
    """Work model per atom (expansion accumulate + 2 flops per harmonic per edge,
    beta transform, power spectrum), with the measured neighbour count."""
    n, L, S = cfg.n_max, cfg.l_max, len(cfg.species)
    H = (L + 1) ** 2
    P = (S * n) * (S * n + 1) // 2
    return edges_per_atom * (2 * n * H + 2 * H) + S * 2 * n * n * H + 2 * P * H


def cpu_baseline(cfg, args, target_seconds=10.0):
    """Reference C++/OpenMP SOAP (oracle/_ref) on a bounded sample of the same workload."""
    sys.path.insert(0, str(ROOT / "oracle"))
    from oracle import RefLib, cpu_threads, reference_available

    from mdescriptor_b200 import workloads
    from mdescriptor_b200.basis import basis_gto

    if not reference_available():
        from oracle import OracleLib

        lib, kind = OracleLib(), "port"
    else:
        lib, kind = RefLib(), "reference"
    threads = cpu_threads()
    alphas, betas = basis_gto(cfg.r_cut, cfg.n_max, cfg.l_max)
    structures = max(threads, 4)
    elapsed, atoms = 0.0, 0
    while True:
        batch = workloads.make(args.config, structures, seed=workloads.SEED_BASE + 900 + args.config)
        t0 = time.perf_counter()
        lib.soap(batch, cfg.species, cfg.r_cut, cfg.n_max, cfg.l_max, cfg.sigma, alphas, betas, cfg.average,
                 num_threads=threads)
        elapsed = time.perf_counter() - t0
        atoms = batch.atoms
        if elapsed >= target_seconds / 4 or structures >= 4096:
            break
        structures = min(4096, int(structures * max(2.0, target_seconds / 4 / max(elapsed, 1e-3))))
    return {"value": atoms / elapsed, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{batch.structures} structures x {batch.atoms // max(batch.structures, 1)} atoms of config "
                      f"{args.config}, {elapsed:.2f} s wall, fp64 output"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from mdescriptor_b200 import workloads

    cfg = workloads.CONFIGS[args.config]
    sys.path.insert(0, str(ROOT / "oracle"))
    from oracle import OracleLib, RefLib, cpu_threads, reference_available

    from mdescriptor_b200.basis import basis_gto

    lib, kind = (RefLib(), "reference") if reference_available() else (OracleLib(), "port")
    threads = cpu_threads()
    alphas, betas = basis_gto(cfg.r_cut, cfg.n_max, cfg.l_max)
    # Bounded per-step sample: enough structures to keep every host thread busy
    # for about 5 s per step.
    structures = max(threads, 4)
    probe = workloads.make(args.config, structures, seed=workloads.SEED_BASE + 900 + args.config)
    t0 = time.perf_counter()
    lib.soap(probe, cfg.species, cfg.r_cut, cfg.n_max, cfg.l_max, cfg.sigma, alphas, betas, cfg.average,
             num_threads=threads)
    per = time.perf_counter() - t0
    structures = int(min(4096, max(structures, structures * 5.0 / max(per, 1e-3))))
    batch = workloads.make(args.config, structures, seed=workloads.SEED_BASE + 900 + args.config)
    for _ in range(args.warmup):
        lib.soap(batch, cfg.species, cfg.r_cut, cfg.n_max, cfg.l_max, cfg.sigma, alphas, betas, cfg.average,
                 num_threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        lib.soap(batch, cfg.species, cfg.r_cut, cfg.n_max, cfg.l_max, cfg.sigma, alphas, betas, cfg.average,
                 num_threads=threads)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = batch.atoms * args.steps / total
    # The GPU arm's config (same workload and shapes); the CPU arm times a
    # bounded sample of it each step, described in cpu_baseline.sample.
    full = workloads.make(args.config, args.structures, seed=rank_seed(args.config, 0))
    ours_config = config_record(args, cfg, full.structures, full.atoms, args.gpus)
    sample = (f"{batch.structures} structures x {batch.atoms // max(batch.structures, 1)} atoms of config "
              f"{args.config} per step")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded generators with the config's shapes; no public dataset)",
        "config": ours_config,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_local(args):
    """One local spectrum (reference default options: cutoff 6, density width
    0.3, max_radial 6, max_angular 4) through the C ABI with host buffers
    (``mdsoap_local_compute``: upload, kernels and the float64 rows' D2H
    inside the host clock), beside the reference's own C++/OpenMP
    ``compute_spherical_expansion`` (oracle/_ref) on a bounded sample."""
    from mdescriptor_b200 import workloads
    from mdescriptor_b200.soap import LOCAL_KINDS, local_feature_count, local_spectrum

    cfg = workloads.CONFIGS[args.config]
    structures = args.structures or 64
    batch = workloads.make(args.config, structures)
    species = list(cfg.species)
    for _ in range(max(1, args.warmup)):
        local_spectrum(args.local, batch, species)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        local_spectrum(args.local, batch, species)
    elapsed = time.perf_counter() - t0
    line = {"metric": f"{args.local} atom-environments/sec", "value": batch.atoms * args.steps / elapsed,
            "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True, "dtype": "f64",
            "path": "mdsoap_local_compute (host buffers: H2D + bin + local_spectra_kernel + D2H per step)",
            "config": {"workload": f"{cfg.name} x {structures} structures", "atoms": batch.atoms,
                       "features": local_feature_count(args.local, species), "cutoff": 6.0, "density_width": 0.3,
                       "max_radial": 6, "max_angular": 4, "output_dtype": "float64"}}
    pkg = ROOT / "oracle" / "_ref" / "pkg"
    if not args.no_cpu_baseline and list(pkg.glob("_native*.so")):
        sys.path.insert(0, str(pkg))
        import _native

        threads = os.cpu_count() or 1
        sample = workloads.make(args.config, max(4, min(structures, threads)), seed=workloads.SEED_BASE + 901)
        t0 = time.perf_counter()
        _native.compute_spherical_expansion(sample.numbers, sample.positions, sample.cells, sample.pbc,
                                            sample.offsets, species, 6.0, 0.3, 6, 4, LOCAL_KINDS[args.local],
                                            2.5, 1, 6.0, threads, None)
        cpu_s = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": sample.atoms / cpu_s, "unit": UNIT, "cores": threads, "kind": "reference",
                                "sample": f"{sample.structures} structures of {cfg.name}, {cpu_s:.2f} s wall"}
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.local:
        run_local(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    import torch

    _, _, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ranks = Ranks("nccl", dev)
    rank, world = ranks.rank, ranks.world

    from mdescriptor_b200 import workloads
    from mdescriptor_b200.basis import basis_gto
    from mdescriptor_b200.soap import Soap, device_view, neighbor_graph, probe_fp64_fma

    cfg = workloads.CONFIGS[args.config]
    batch = workloads.make(args.config, args.structures, seed=rank_seed(args.config, rank))
    alphas, betas = basis_gto(cfg.r_cut, cfg.n_max, cfg.l_max)
    soap = Soap(cfg.species, r_cut=cfg.r_cut, n_max=cfg.n_max, l_max=cfg.l_max, sigma=cfg.sigma,
                average=cfg.average, dtype=cfg.dtype, alphas=alphas, betas=betas)
    rows = soap.rows(batch)
    out_dtype = torch.float32 if cfg.dtype == "float32" else torch.float64
    elem = 4 if cfg.dtype == "float32" else 8
    atoms_all = ranks.sum(batch.atoms)
    rows_all = ranks.sum(rows)

    sampler = ClockSampler(local)
    sampler.start()

    # ---- device-resident value
    names = ("numbers", "positions", "cells", "pbc", "offsets")
    tensors = [torch.from_numpy(np.ascontiguousarray(getattr(batch, k))).to(dev) for k in names]
    out = torch.empty((rows, soap.feature_count), dtype=out_dtype, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    view = device_view(*(t.data_ptr() for t in tensors), batch.structures, batch.atoms)
    stream = torch.cuda.current_stream(dev)
    soap.set_timing(True)
    for _ in range(args.warmup):
        flush.fill_(1)
        soap.compute_device(view, out.data_ptr(), local, stream.cuda_stream)
    soap.check(local, stream.cuda_stream)
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    center_ms, bin_ms, expansion_ms, tail_ms = [], [], [], []
    ranks.barrier()
    torch.cuda.synchronize(dev)
    launches0 = soap.launch_count()
    sampler.begin()
    for start, stop in events:
        flush.fill_(1)
        start.record(stream)
        soap.compute_device(view, out.data_ptr(), local, stream.cuda_stream)
        stop.record(stream)
        b, c, _ = soap.last_timing(local)
        bin_ms.append(b)
        center_ms.append(c)
        x, t = soap.last_timing_split(local)
        expansion_ms.append(x)
        tail_ms.append(t)
    torch.cuda.synchronize(dev)
    sampler.end()
    ranks.barrier()
    soap.check(local, stream.cuda_stream)
    total_ms = ranks.max(sum(s.elapsed_time(e) for s, e in events))
    value = job_throughput(atoms_all, args.steps, total_ms)
    gpu_launches = soap.launch_count() - launches0
    launches_per_step = gpu_launches / args.steps

    # ---- end to end through the public host API (pinned host buffers)
    e2e = None
    if not args.no_e2e:
        pinned = {}
        for k in names:
            host = np.ascontiguousarray(getattr(batch, k))
            t = torch.empty(host.shape, dtype=torch.from_numpy(host).dtype, pin_memory=True)
            t.numpy()[...] = host
            pinned[k] = t.numpy()
        pbatch = workloads.Batch(*(pinned[k] for k in names))
        host_out = torch.empty((rows, soap.feature_count), dtype=out_dtype, pin_memory=True).numpy()
        for _ in range(max(1, args.warmup)):
            soap.compute(pbatch, devices=[local], out=host_out)
        ranks.barrier()
        torch.cuda.synchronize(dev)
        launches1 = soap.launch_count()
        sampler.begin()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            soap.compute(pbatch, devices=[local], out=host_out)
        torch.cuda.synchronize(dev)
        e2e_s = time.perf_counter() - t0
        sampler.end()
        ranks.barrier()
        e2e_s = ranks.max(e2e_s)
        h2d = ranks.sum(sum(pinned[k].nbytes for k in names))
        e2e = {"value": job_throughput(atoms_all, args.steps, e2e_s * 1e3), "unit": UNIT,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(rows_all * soap.feature_count * elem),
               "path": "Soap.compute (C ABI mdsoap_compute): pinned host in/out, H2D + kernels + D2H per step; "
                       "host clock around synchronous calls, synchronize + barrier on both sides, max over ranks"}
        e2e["gpu_launches"] = soap.launch_count() - launches1
    clocks = sampler.stop()

    if rank == 0:
        # measured neighbour count (edges per atom incl. self) on a sample
        sample = batch.slice(0, min(batch.structures, 16))
        g = neighbor_graph(sample, soap.cutoff, local)
        edges = len(g[1]) / max(sample.atoms, 1)
        center_avg_s = statistics.mean(center_ms) * 1e-3
        bytes_per_launch = batch.atoms * (4 + 24 + rows / batch.atoms * soap.feature_count * elem)
        hbm_peak, hbm_src = measured_peaks()
        achieved_gbs = bytes_per_launch / center_avg_s / 1e9
        traffic = None
        kernel = soap.kernel()
        tf = ROOT / "profiles" / f"traffic_config{args.config}.json"
        if tf.is_file():
            # one-pass ncu capture of the full-size launch (dram read + write)
            # of the same kernel; other sizes scale it by atoms (the rows are
            # the traffic)
            record = json.loads(tf.read_text())
            if record.get("kernel") == kernel:
                traffic = record["dram_bytes_per_launch"] * batch.atoms / record["atoms"]
        fp64_peak = probe_fp64_fma(local)
        flops = algorithmic_flops_per_atom(cfg, edges) * batch.atoms
        achieved_tf = flops / center_avg_s / 1e12
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded generators with the config's shapes; no public dataset)",
            "config": config_record(args, cfg, batch.structures, batch.atoms, world),
            "e2e": e2e,
            "gpu_launches": gpu_launches,
            "gpu_launches_per_step": launches_per_step,
            "kernel_ms": {"bin": statistics.mean(bin_ms), "center": statistics.mean(center_ms),
                          "expansion": statistics.mean(expansion_ms), "tail": statistics.mean(tail_ms)},
            "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved_gbs / hbm_peak, "traffic": traffic,
                         "kernel": kernel, "peak_source": hbm_src,
                         "algorithmic_bytes_per_atom": bytes_per_launch / batch.atoms},
            "roofline_fp64": {"bound": "fp64", "achieved": achieved_tf, "peak": fp64_peak, "unit": "TFLOP/s",
                              "frac": achieved_tf / fp64_peak, "kernel": kernel,
                              "peak_source": "measured in-run (mdsoap_probe_fp64_fma, FMA chains on every SM)",
                              "flops_per_atom": flops / batch.atoms, "edges_per_atom": edges,
                              "exp_per_atom": edges * (cfg.l_max + 1) * cfg.n_max},
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg, args)
        print(json.dumps(line), flush=True)
    ranks.close()


if __name__ == "__main__":
    main()
