#!/usr/bin/env python
"""SOAP atom-environments/s on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 5] [--impl ours|reference]

A step is one pass of the SOAP hot path (neighbour search, expansion, power
spectrum) over one seeded batch of synthetic structures with the shape of the
chosen benchmark config.  The default is config 5, the one the metric's
1/2/4/8-GPU sweep names: 65 536 periodic 16 A cells x 256 atoms (16.8 M atom
environments), species 1/6/8, r_cut 5.5, n_max 8, l_max 6, float32 rows.
With N ranks (torchrun, one process per GPU), rank r computes structures
[r S / N, (r + 1) S / N) of that one batch: strong scaling, no exchange step.

* ``value``: device-resident throughput -- the shard's inputs already in HBM,
  its rows written to HBM (141 GB of float32 rows at N = 1), CUDA events on
  the launching stream around each step, L2 flushed (256 MiB write) between
  steps outside the events; all ranks' atoms over the slowest rank's time.
* ``e2e``: the same metric through the host C ABI (``Soap.compute``):
  pinned host inputs uploaded and every output row copied back to pinned host
  memory inside the timed region, on the leading slice of each shard whose
  rows fit a pinned host buffer.
* ``e2e_api``: the same metric through the reference's unchanged public API
  (``SOAP(...).compute`` with ``device="cuda"``, staged in baseline/_ref),
  which reaches this repository's plugin through MDESCRIPTOR_CUDA_PLUGIN_DIR.
* ``sharder_check`` (N > 1): rank 0 runs the in-process multi-device sharder
  (``mdsoap_compute`` over every GPU of the job) and compares its rows bitwise
  with one device's.
* ``roofline``: the expansion + tail kernels against the measured HBM copy
  bandwidth (compulsory bytes), plus ``roofline_fp64`` against the measured
  fp64 FMA rate.
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
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--config", type=int, default=5)
    p.add_argument("--structures", type=int, default=None,
                   help="structures of the whole batch, shared by the ranks (default: the config's)")
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-api", action="store_true", help="skip the reference public-API figure (e2e_api)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--local", default=None, choices=("SphericalExpansion", "SoapRadialSpectrum", "SoapPowerSpectrum"),
                   help="time a local spherical spectrum (reference defaults) instead of SOAP; one GPU")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def smi_device_id(local: int) -> str:
    """nvidia-smi's identifier of CUDA device `local`: the CUDA_VISIBLE_DEVICES
    entry when that is set (an index or a UUID, both of which --id accepts),
    else the index itself."""
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "").strip()
    if visible:
        entries = [e.strip() for e in visible.split(",") if e.strip()]
        if local < len(entries):
            return entries[local]
    return str(local)


def parse_cpulist(text: str) -> set[int]:
    """CPUs of a sysfs cpulist ("0-15,32-47")."""
    cpus: set[int] = set()
    for part in text.strip().split(","):
        if not part:
            continue
        lo, _, hi = part.partition("-")
        cpus.update(range(int(lo), int(hi or lo) + 1))
    return cpus


def bind_to_gpu_node(pci_address: str, sysfs: Path = Path("/sys")) -> dict:
    """Restrict this process to the CPUs of its GPU's NUMA node, so that the
    page-locked host buffers it touches first (rows, staging) are allocated on
    the node the GPU's PCIe link attaches to.  A GPU without a node (-1, as in
    single-node guests) or an unreadable sysfs leaves the affinity as it is."""
    try:
        node = int((sysfs / "bus/pci/devices" / pci_address / "numa_node").read_text())
    except (OSError, ValueError):
        return {"numa_node": None, "cpus": "unchanged (no sysfs record)"}
    if node < 0:
        return {"numa_node": None, "cpus": "unchanged (single node)"}
    try:
        text = (sysfs / f"devices/system/node/node{node}/cpulist").read_text().strip()
        cpus = parse_cpulist(text) & os.sched_getaffinity(0)
    except (OSError, ValueError):
        return {"numa_node": node, "cpus": "unchanged (no cpulist)"}
    if not cpus:
        return {"numa_node": node, "cpus": "unchanged (no allowed CPU on the node)"}
    os.sched_setaffinity(0, cpus)
    return {"numa_node": node, "cpus": text}


# Structures of each config's full batch, and atoms per
# structure where that is fixed.
DEFAULT_STRUCTURES = {1: 64, 2: 1024, 3: 8, 4: 16384, 5: 65536}
ATOMS_PER_STRUCTURE = {1: 64, 2: 128, 3: 32768, 5: 256}


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Structures [r S / N, (r + 1) S / N) of the batch belong to rank r."""
    return total * rank // world, total * (rank + 1) // world


def shard_batch(config: int, total: int, rank: int, world: int):
    """This rank's contiguous structure range of the config's one seeded batch.
    Config 5 generates only the shard (per-structure streams); the smaller
    configs generate the whole batch and slice it."""
    from mdescriptor_b200 import workloads

    s0, s1 = shard_range(total, rank, world)
    if config == 5:
        return workloads.make(5, s1 - s0, first=s0)
    return workloads.make(config, total).slice(s0, s1)


class Ranks:
    """One process per GPU, launched by torchrun (RANK/WORLD_SIZE/LOCAL_RANK).

    The only collectives are a barrier around the timed regions and the
    max / sum reductions of the per-rank timings and unit counts -- the SOAP
    path itself shards by structure with no exchange.  ``backend`` is "nccl"
    on GPUs and "gloo" for the CPU tests of this logic.
    """

    def __init__(self, backend: str = "nccl", device=None, timeout_s: float = 300.0):
        self.rank, self.world, self.local = dist_env()
        self.device = device
        self.group = None
        self.host_group = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            kwargs = {"device_id": device} if backend == "nccl" else {}
            timeout = datetime.timedelta(seconds=timeout_s)
            dist.init_process_group(backend, timeout=timeout, **kwargs)
            self.group = dist
            # A host-side group: ranks that wait for rank 0's multi-device
            # work wait on the CPU, with no kernel of theirs on the GPUs.
            self.host_group = dist.new_group(backend="gloo", timeout=timeout) if backend != "gloo" else None

    def barrier(self):
        if self.group is not None:
            self.group.barrier()

    def host_barrier(self):
        if self.group is not None:
            self.group.barrier(group=self.host_group)

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

    def min(self, x: float) -> float:
        return self._reduce(x, None if self.group is None else self.group.ReduceOp.MIN)

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
        "structures": structures,
        "atoms": atoms,
        "species": list(cfg.species),
        "r_cut": cfg.r_cut,
        "n_max": cfg.n_max,
        "l_max": cfg.l_max,
        "sigma": cfg.sigma,
        "average": cfg.average,
        "output_dtype": cfg.dtype,
        "parallelism": parallelism or f"one batch sharded by structure over {world} GPU(s) (no collective)",
        "l2": "flushed between steps (256 MiB device write, outside the timed events); the rows of a step "
              "are also far larger than L2",
    }


def scaled_traffic(config: int, kernel: str, atoms: int):
    """DRAM bytes (read + write) per step of the expansion + tail kernels,
    scaled by atoms from a committed ncu capture of a small case of the same
    kernels (profiles/traffic_config<k>.json: one kernel per capture, a few
    launches, inputs and rows larger than L2).  The traffic is the rows and
    the raw-sum round trip, both proportional to atoms."""
    path = ROOT / "profiles" / f"traffic_config{config}.json"
    if not path.is_file():
        return None, None
    record = json.loads(path.read_text())
    if record.get("kernel") != kernel:
        return None, None
    return record["dram_bytes_per_launch"] * atoms / record["atoms"], f"{path.name} (scaled by atoms)"


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

    def __init__(self, device: str):
        self.device = device  # nvidia-smi --id value
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
    elapsed = sum(times)
    value = batch.atoms * args.steps / elapsed
    # The GPU arm's config (same workload and shapes); the CPU arm times a
    # bounded sample of it each step, described in cpu_baseline.sample.
    total = args.structures or DEFAULT_STRUCTURES[args.config]
    atoms_total = (total * ATOMS_PER_STRUCTURE[args.config] if args.config in ATOMS_PER_STRUCTURE
                   else workloads.make(args.config, total).atoms)
    ours_config = config_record(args, cfg, total, atoms_total, args.gpus)
    ours_config["workload"] += f": one seeded batch of {total} structures"
    if args.gpus > 1:
        ours_config["workload"] += f", sharded by structure over {args.gpus} ranks"
    sample = (f"{batch.structures} structures x {batch.atoms // max(batch.structures, 1)} atoms of config "
              f"{args.config} per step")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
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


def device_memory_fit(soap, cfg, batch, rows, elem, dev) -> tuple[int, dict]:
    """Largest leading slice of this rank's shard whose device working set fits:
    the rows, the engine's per-atom workspace (inputs, bins, sorted positions),
    the split tail's raw-sum chunk and edge slots (4 GiB each at most) and
    the L2 flush buffer, with 2 GiB spare."""
    import torch

    free, total = torch.cuda.mem_get_info(dev)
    per_atom = rows / max(batch.atoms, 1) * soap.feature_count * elem + 160
    fixed = (9 << 30) + L2_FLUSH_BYTES + (2 << 30)
    fit_atoms = int(max(0, free - fixed) // per_atom)
    structures = batch.structures
    if fit_atoms < batch.atoms:
        structures = max(1, int(np.searchsorted(batch.offsets, fit_atoms, side="right")) - 1)
    return structures, {"device_free_gib": round(free / 2**30, 1), "device_total_gib": round(total / 2**30, 1)}


def host_memory_available() -> int:
    try:
        for line in Path("/proc/meminfo").read_text().splitlines():
            if line.startswith("MemAvailable:"):
                return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 16 << 30


def e2e_structures(batch, rows_per_structure_bytes: float, world: int, cap_bytes: int = 8 << 30) -> int:
    """Structures of this rank's shard timed end to end: the whole shard when
    its rows fit a pinned host buffer of min(8 GiB, a quarter of the host's
    available memory shared by the ranks), else the largest leading slice
    that does."""
    budget = min(cap_bytes, host_memory_available() // (4 * max(world, 1)))
    fit = int(budget // max(rows_per_structure_bytes, 1.0))
    return max(1, min(batch.structures, fit))


def api_path_throughput(cfg, batch, steps, local, ranks, sampler):
    """The same metric through the reference's unchanged public API:
    ``SOAP(..., execution=ExecutionOptions(device="cuda")).compute(StructureBatch)``
    from the reference package staged in baseline/_ref, with
    MDESCRIPTOR_CUDA_PLUGIN_DIR pointing at this repository's plugin.  The
    adapter calls the plugin once per 32-structure block (pageable NumPy rows
    from each call) and concatenates the blocks; all of it is inside the host
    clock.  Returns None when the reference package is not staged."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "mdescriptor" / "__init__.py").is_file():
        return None
    os.environ["MDESCRIPTOR_CUDA_PLUGIN_DIR"] = str(ROOT / "mdescriptor_b200" / "plugin")
    os.environ["MDSOAP_DEVICES"] = str(local)  # the plugin's device selector: this rank's GPU
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    from mdescriptor import ExecutionOptions, OutputOptions, StructureBatch
    from mdescriptor._cuda_loader import load_cuda_plugin
    from mdescriptor.descriptors import SOAP

    import torch

    # The reference loads its CUDA plugin on request (its own tests and
    # benchmarks call this loader, which honours MDESCRIPTOR_CUDA_PLUGIN_DIR).
    load_cuda_plugin()

    sb = StructureBatch(batch.numbers, batch.positions, batch.cells, batch.pbc, batch.offsets,
                        tuple(f"s{i}" for i in range(batch.structures)))
    soap = SOAP(species=list(cfg.species), r_cut=cfg.r_cut, n_max=cfg.n_max, l_max=cfg.l_max, sigma=cfg.sigma,
                average=cfg.average, output=OutputOptions(dtype=cfg.dtype), execution=ExecutionOptions(device="cuda"))
    result = soap.compute(sb)  # warm-up (loads the plugin, builds the backend)
    rows = int(np.asarray(result.values).shape[0])
    del result
    ranks.barrier()
    torch.cuda.synchronize()
    sampler.begin()
    t0 = time.perf_counter()
    for _ in range(steps):
        result = soap.compute(sb)
        del result
    elapsed = time.perf_counter() - t0
    sampler.end()
    ranks.barrier()
    return elapsed, rows


def main():
    args = parse_args()
    if args.local:
        run_local(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    import torch

    _, world_env, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    host_binding = None
    if world_env > 1:
        # Several ranks share the host: keep each one's page-locked buffers on
        # its GPU's NUMA node (N = 1 keeps every core for the CPU baseline).
        props = torch.cuda.get_device_properties(local)
        host_binding = bind_to_gpu_node(
            f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0")
    ranks = Ranks("nccl", dev)
    rank, world = ranks.rank, ranks.world

    from mdescriptor_b200 import workloads
    from mdescriptor_b200.basis import basis_gto
    from mdescriptor_b200.soap import Soap, device_view, neighbor_graph, probe_fp64_fma

    cfg = workloads.CONFIGS[args.config]
    total_structures = args.structures or DEFAULT_STRUCTURES[args.config]
    s0, s1 = shard_range(total_structures, rank, world)
    batch = shard_batch(args.config, total_structures, rank, world)
    alphas, betas = basis_gto(cfg.r_cut, cfg.n_max, cfg.l_max)
    soap = Soap(cfg.species, r_cut=cfg.r_cut, n_max=cfg.n_max, l_max=cfg.l_max, sigma=cfg.sigma,
                average=cfg.average, dtype=cfg.dtype, alphas=alphas, betas=betas)
    out_dtype = torch.float32 if cfg.dtype == "float32" else torch.float64
    elem = 4 if cfg.dtype == "float32" else 8

    # The whole shard device-resident when it fits; else the largest leading
    # slice (recorded in config.workload).
    fit_structures, memory = device_memory_fit(soap, cfg, batch, soap.rows(batch), elem, dev)
    fitted = ranks.min(fit_structures) >= batch.structures
    if fit_structures < batch.structures:
        batch = batch.slice(0, fit_structures)
    rows = soap.rows(batch)
    atoms_all = ranks.sum(batch.atoms)
    structures_all = ranks.sum(batch.structures)

    sampler = ClockSampler(smi_device_id(local))
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
    gpu_launches = int(ranks.sum(soap.launch_count() - launches0))
    del out, flush, tensors

    # ---- end to end through the host C ABI (pinned host buffers)
    e2e = None
    e2e_batch = batch.slice(0, e2e_structures(batch, soap.rows(batch.slice(0, 1)) * soap.feature_count * elem, world))
    pinned = {}
    for k in names:
        host = np.ascontiguousarray(getattr(e2e_batch, k))
        t = torch.empty(host.shape, dtype=torch.from_numpy(host).dtype, pin_memory=True)
        t.numpy()[...] = host
        pinned[k] = t.numpy()
    pbatch = workloads.Batch(*(pinned[k] for k in names))
    e2e_rows = soap.rows(pbatch)
    host_out = torch.empty((e2e_rows, soap.feature_count), dtype=out_dtype, pin_memory=True).numpy()
    if not args.no_e2e:
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
        e2e_atoms = ranks.sum(pbatch.atoms)
        h2d = ranks.sum(sum(pinned[k].nbytes for k in names))
        d2h = ranks.sum(e2e_rows * soap.feature_count * elem)
        e2e = {"value": job_throughput(e2e_atoms, args.steps, e2e_s * 1e3), "unit": UNIT,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "structures_per_rank": pbatch.structures,
               "path": "Soap.compute (C ABI mdsoap_compute): pinned host in/out, H2D + kernels + D2H per step, "
                       "on the leading slice of each rank's shard whose rows fit a pinned host buffer of "
                       "min(8 GiB, a quarter of the host's available memory / ranks); host clock around "
                       "synchronous calls, synchronize + barrier on both sides, max over ranks",
               "gpu_launches": int(ranks.sum(soap.launch_count() - launches1))}

    # ---- the same metric through the reference's unchanged public API
    e2e_api = None
    if not args.no_e2e and not args.no_api:
        api_batch = batch.slice(0, min(batch.structures, 512))
        got = api_path_throughput(cfg, api_batch, max(1, min(args.steps, 5)), local, ranks, sampler)
        if got is not None:
            api_s, api_rows = got
            api_s = ranks.max(api_s)
            steps = max(1, min(args.steps, 5))
            e2e_api = {"value": job_throughput(ranks.sum(api_batch.atoms), steps, api_s * 1e3), "unit": UNIT,
                       "steps": steps, "structures_per_rank": api_batch.structures,
                       "d2h_bytes_per_step": int(ranks.sum(api_rows * soap.feature_count * elem)),
                       "path": "reference SOAP(..., ExecutionOptions(device='cuda')).compute(StructureBatch) "
                               "(baseline/_ref) -> mdescriptor._cuda plugin (MDESCRIPTOR_CUDA_PLUGIN_DIR): "
                               "32-structure blocks, pageable NumPy rows, block concatenation; host clock, "
                               "max over ranks"}

    # ---- the in-process multi-device sharder (mdsoap_compute with every
    # device of the job) on rank 0, checked bitwise against one device
    sharder = None
    if world > 1:
        if rank == 0:
            try:
                single = soap.compute(pbatch, devices=[0])
                t0 = time.perf_counter()
                multi = soap.compute(pbatch, devices=list(range(world)))
                sharder_s = time.perf_counter() - t0
                sharder = {"devices": world, "structures": pbatch.structures,
                           "bitwise_equal_to_one_device": bool(np.array_equal(single, multi)),
                           "seconds": sharder_s}
                del single, multi
            except Exception as exc:  # reported, not raised: the other ranks wait for rank 0
                sharder = {"devices": world, "error": f"{type(exc).__name__}: {exc}"}
        ranks.host_barrier()
    clocks = sampler.stop()

    if rank == 0:
        # measured neighbour count (edges per atom incl. self) on a sample
        sample = batch.slice(0, min(batch.structures, 16))
        g = neighbor_graph(sample, soap.cutoff, local)
        edges = len(g[1]) / max(sample.atoms, 1)
        center_avg_s = statistics.mean(center_ms) * 1e-3
        bytes_per_atom = 4 + 24 + rows / batch.atoms * soap.feature_count * elem
        bytes_per_launch = batch.atoms * bytes_per_atom
        hbm_peak, hbm_src = measured_peaks()
        achieved_gbs = bytes_per_launch / center_avg_s / 1e9
        kernel = soap.kernel()
        traffic, traffic_src = scaled_traffic(args.config, kernel, batch.atoms)
        fp64_peak = probe_fp64_fma(local)
        flops = algorithmic_flops_per_atom(cfg, edges) * batch.atoms
        achieved_tf = flops / center_avg_s / 1e12
        workload = f"{cfg.name} (BASELINE config {args.config}): one seeded batch of {total_structures} structures"
        if world > 1:
            workload += f", sharded by structure over {world} ranks"
        if not fitted:
            workload += (f"; the device-resident timing covers the leading {structures_all} structures that fit "
                         f"the ranks' HBM")
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded generators with the config's shapes; no public dataset)",
            "config": dict(config_record(args, cfg, structures_all, atoms_all, world), workload=workload,
                           structures_total=total_structures, structures_per_rank=batch.structures,
                           atoms_per_rank=batch.atoms, shard=[s0, s0 + batch.structures], **memory),
            "e2e": e2e,
            "e2e_api": e2e_api,
            "gpu_launches": gpu_launches,
            "gpu_launches_per_step": gpu_launches / args.steps,
            "kernel_ms": {"bin": statistics.mean(bin_ms), "center": statistics.mean(center_ms),
                          "expansion": statistics.mean(expansion_ms), "tail": statistics.mean(tail_ms)},
            "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved_gbs / hbm_peak, "traffic": traffic, "traffic_source": traffic_src,
                         "kernel": kernel, "peak_source": hbm_src,
                         "algorithmic_bytes_per_atom": bytes_per_atom},
            "roofline_fp64": {"bound": "fp64", "achieved": achieved_tf, "peak": fp64_peak, "unit": "TFLOP/s",
                              "frac": achieved_tf / fp64_peak, "kernel": kernel,
                              "peak_source": "measured in-run (mdsoap_probe_fp64_fma, FMA chains on every SM)",
                              "flops_per_atom": flops / batch.atoms, "edges_per_atom": edges,
                              "exp_per_atom": edges * (cfg.l_max + 1) * cfg.n_max},
            "clocks": clocks,
        }
        if sharder is not None:
            line["sharder_check"] = sharder
        if host_binding is not None:
            line["config"]["host_binding"] = host_binding
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg, args)
        print(json.dumps(line), flush=True)
    ranks.close()


if __name__ == "__main__":
    main()
