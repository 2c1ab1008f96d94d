"""Config 5 at full size on one GPU: 65 536 periodic 16 A cells x 256 atoms
(16.8 M atom environments, 141 GB of float32 rows), device-resident through
the C ABI (``mdsoap_compute_device``), the batch the benchmark times.

* sampled structures from the whole range against the reference's own CPU
  SOAP (``oracle/_ref/libref_soap.so``, compiled from its sources), within
  the float32 bound;
* size-independent properties: every row finite, and three structure ranges
  recomputed on their own equal the full run's rows bit for bit (structures
  are independent, and a step's chunking of the work does not change a
  row's arithmetic).
"""

from __future__ import annotations

import numpy as np
import pytest

from _util import assert_features_close
from mdescriptor_b200 import workloads
from mdescriptor_b200.basis import basis_gto
from mdescriptor_b200.soap import Soap, device_view

pytestmark = pytest.mark.gpu

SAMPLE = (0, 1, 4097, 20000, 32767, 32768, 51234, 65535)
RANGES = ((0, 3), (30000, 30512), (65530, 65536))


def _checker():
    from oracle import OracleLib, RefLib, reference_available

    return RefLib() if reference_available() else OracleLib()


def test_config5_full_batch_on_one_gpu(cuda_device):
    import torch

    cfg = workloads.CONFIGS[5]
    batch = workloads.config5()
    alphas, betas = basis_gto(cfg.r_cut, cfg.n_max, cfg.l_max)
    soap = Soap(cfg.species, r_cut=cfg.r_cut, n_max=cfg.n_max, l_max=cfg.l_max, sigma=cfg.sigma, average="off",
                dtype="float32", alphas=alphas, betas=betas)
    rows, F = batch.atoms, soap.feature_count
    dev = torch.device("cuda", cuda_device)
    free, _ = torch.cuda.mem_get_info(dev)
    need = rows * F * 4 + (8 << 30)
    if free < need:
        pytest.skip(f"config 5 needs {need / 2**30:.0f} GiB of free device memory; {free / 2**30:.0f} GiB free")
    names = ("numbers", "positions", "cells", "pbc", "offsets")
    tensors = [torch.from_numpy(np.ascontiguousarray(getattr(batch, k))).to(dev) for k in names]
    out = torch.empty((rows, F), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    try:
        soap.compute_device(device_view(*(t.data_ptr() for t in tensors), batch.structures, batch.atoms),
                            out.data_ptr(), cuda_device, stream)
        soap.check(cuda_device, stream)
        chunk = 1 << 20
        for r0 in range(0, rows, chunk):
            assert bool(torch.isfinite(out[r0:r0 + chunk]).all()), f"non-finite rows in [{r0}, {r0 + chunk})"
        # sampled structures against the reference CPU path
        checker = _checker()
        for s in SAMPLE:
            one = batch.slice(s, s + 1)
            got = out[s * 256:(s + 1) * 256].cpu().numpy()
            want = checker.soap(one, cfg.species, cfg.r_cut, cfg.n_max, cfg.l_max, cfg.sigma, alphas, betas, "off")
            assert_features_close(got, want, np.float32)
        # structure ranges on their own: bit for bit the full run's rows
        for s0, s1 in RANGES:
            part = batch.slice(s0, s1)
            pt = [torch.from_numpy(np.ascontiguousarray(getattr(part, k))).to(dev) for k in names]
            pout = torch.empty((part.atoms, F), dtype=torch.float32, device=dev)
            soap.compute_device(device_view(*(t.data_ptr() for t in pt), part.structures, part.atoms),
                                pout.data_ptr(), cuda_device, stream)
            soap.check(cuda_device, stream)
            assert torch.equal(pout, out[s0 * 256:s1 * 256]), f"structures [{s0}, {s1}) differ from the full run"
    finally:
        del out, tensors
        soap.close()
        torch.cuda.empty_cache()
