"""bench.py's multi-rank logic on CPU: world_size-2 ``gloo`` ranks.

The SOAP path shards one batch by structure with no data exchange, so the
only collectives are the barrier and the max / sum reductions around the
timed regions; these tests run exactly those helpers on two processes, plus
the shard arithmetic and the reference arm's "rank 0 alone works" rule.
"""

from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    ranks = bench.Ranks("gloo", None, timeout_s=30)
    try:
        ranks.barrier()
        local_ms = 10.0 * (rank + 1)        # rank 1 is the slow one
        local_atoms = 100 + 28 * rank       # ragged shards
        total_ms = ranks.max(local_ms)
        atoms_all = ranks.sum(local_atoms)
        value = bench.job_throughput(atoms_all, 4, total_ms)
        queue.put((rank, ranks.world, total_ms, atoms_all, value, bench.shard_range(65536, rank, world)))
    finally:
        ranks.close()


def test_two_gloo_ranks_take_max_time_and_sum_units():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, w0, t0, a0, v0, s0), (r1, w1, t1, a1, v1, s1) = results
    assert (r0, r1, w0, w1) == (0, 1, 2, 2)
    assert t0 == t1 == 20.0                       # max over ranks
    assert a0 == a1 == 228                        # units of all ranks
    assert v0 == v1 == pytest.approx(228 * 4 / 0.020)
    assert s0 == (0, 32768) and s1 == (32768, 65536)  # one batch, contiguous shards


def test_shards_cover_the_batch_once_and_slice_the_one_seeded_batch():
    import numpy as np

    from mdescriptor_b200 import workloads

    for world in (1, 2, 3, 4, 8):
        ranges = [bench.shard_range(65536, r, world) for r in range(world)]
        assert ranges[0][0] == 0 and ranges[-1][1] == 65536
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    whole = workloads.make(5, 12)
    for world in (2, 3):
        parts = [bench.shard_batch(5, 12, r, world) for r in range(world)]
        np.testing.assert_array_equal(np.concatenate([p.positions for p in parts]), whole.positions)
        np.testing.assert_array_equal(np.concatenate([p.numbers for p in parts]), whole.numbers)
    small = [bench.shard_batch(1, 8, r, 2) for r in range(2)]
    np.testing.assert_array_equal(np.concatenate([p.positions for p in small]), workloads.make(1, 8).positions)


def test_e2e_slice_respects_the_host_budget(monkeypatch):
    from mdescriptor_b200 import workloads

    batch = workloads.make(5, 64)
    monkeypatch.setattr(bench, "host_memory_available", lambda: 64 << 30)
    row_bytes = 256 * 2100 * 4  # one structure's float32 rows
    assert bench.e2e_structures(batch, row_bytes, 1) == 64          # the whole shard fits
    assert bench.e2e_structures(batch, row_bytes, 1, cap_bytes=10 * row_bytes) == 10
    monkeypatch.setattr(bench, "host_memory_available", lambda: 4 * 8 * 5 * row_bytes)
    assert bench.e2e_structures(batch, row_bytes, 8) == 5            # a quarter of the host, shared by 8 ranks


def test_single_process_ranks_are_identity():
    for key in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        os.environ.pop(key, None)
    ranks = bench.Ranks("gloo")
    assert (ranks.rank, ranks.world, ranks.group) == (0, 1, None)
    assert ranks.max(3.5) == 3.5 and ranks.sum(7) == 7.0 and ranks.min(2.0) == 2.0
    ranks.barrier()
    ranks.host_barrier()
    ranks.close()


def test_reference_arm_runs_on_rank_zero_only():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2"],
                         env=env, capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == ""


def test_clock_summary_keeps_only_samples_inside_timed_windows():
    samples = [(0.5, "600, 1965, 100.0, Not Active, Not Active, Not Active, Not Active"),
               (1.5, "1900, 1965, 900.0, Not Active, Not Active, Not Active, Active"),
               (1.7, "1800, 1965, 950.0, Not Active, Not Active, Not Active, Not Active"),
               (3.0, "500, 1965, 90.0, Active, Not Active, Not Active, Not Active")]
    summary = bench.summarize_clocks(samples, [[1.0, 2.0]])
    assert summary["samples"] == 2
    assert summary["sm_mhz"] == 1850.0 and summary["sm_max_mhz"] == 1965.0
    assert summary["reasons"] == ["sw_power_cap"]
    assert bench.summarize_clocks(samples, [[10.0, 11.0]]) is None


def test_ranks_bind_to_their_gpus_numa_node(tmp_path, monkeypatch):
    """Each rank of a multi-GPU run restricts itself to the CPUs of its GPU's
    NUMA node (read from a fake sysfs tree here); a node of -1 or a missing
    record leaves the affinity alone."""
    assert bench.parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    allowed = sorted(os.sched_getaffinity(0))
    dev = tmp_path / "bus/pci/devices/0000:18:00.0"
    dev.mkdir(parents=True)
    node = tmp_path / "devices/system/node/node1"
    node.mkdir(parents=True)
    (node / "cpulist").write_text(f"{allowed[0]}-{allowed[0]}\n")
    calls = []
    monkeypatch.setattr(bench.os, "sched_setaffinity", lambda pid, cpus: calls.append(set(cpus)))

    (dev / "numa_node").write_text("1\n")
    assert bench.bind_to_gpu_node("0000:18:00.0", tmp_path) == {"numa_node": 1, "cpus": f"{allowed[0]}-{allowed[0]}"}
    assert calls == [{allowed[0]}]

    (dev / "numa_node").write_text("-1\n")
    assert bench.bind_to_gpu_node("0000:18:00.0", tmp_path)["numa_node"] is None
    assert bench.bind_to_gpu_node("0000:99:00.0", tmp_path)["numa_node"] is None
    assert len(calls) == 1


def test_clock_sampler_follows_visible_devices(monkeypatch):
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    assert bench.smi_device_id(3) == "3"
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "5,GPU-0a1b2c3d-0000-1111-2222-333344445555")
    assert bench.smi_device_id(0) == "5"
    assert bench.smi_device_id(1) == "GPU-0a1b2c3d-0000-1111-2222-333344445555"


def test_reference_arm_line_is_consistent():
    """The reference arm's ms_per_step is the time of one timed step of its
    sample: value x ms_per_step equals the sample's atoms."""
    import json
    import re

    if not (ROOT / "oracle" / "_ref" / "libref_soap.so").exists() and not (ROOT / "oracle" / "liboracle_soap.so").exists():
        pytest.skip("no CPU checker built")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--config", "1",
                          "--steps", "1", "--warmup", "0"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr
    line = json.loads(out.stdout.strip().splitlines()[-1])
    structures, atoms = map(int, re.match(r"(\d+) structures x (\d+) atoms", line["cpu_baseline"]["sample"]).groups())
    assert line["impl"] == "reference" and line["steps"] == 1
    assert abs(line["value"] * line["ms_per_step"] / 1e3 - structures * atoms) <= 0.01 * structures * atoms
