"""A small, fixed SOAP case for profiler captures (``ncu``): the leading
structures of a benchmark config computed device-resident through the C ABI
(``mdsoap_compute_device``), a few times, with nothing else on the GPU.

    python -m mdescriptor_b200.profile_case --config 5 --structures 512 --repeats 2

The default, 512 config-5 cells (131 072 atoms, 1.1 GB of float32 rows), is
larger than L2, so DRAM counters mean what they do at full size, and small
enough for a full ncu capture of one launch to end in a minute or two.
"""

from __future__ import annotations

import argparse


def main() -> None:
    import numpy as np
    import torch

    from . import workloads
    from .basis import basis_gto
    from .soap import Soap, device_view

    p = argparse.ArgumentParser()
    p.add_argument("--config", type=int, default=5)
    p.add_argument("--structures", type=int, default=512)
    p.add_argument("--repeats", type=int, default=2)
    p.add_argument("--dtype", default=None, help="override the config's output dtype")
    args = p.parse_args()
    cfg = workloads.CONFIGS[args.config]
    batch = workloads.make(args.config, args.structures)
    alphas, betas = basis_gto(cfg.r_cut, cfg.n_max, cfg.l_max)
    dtype = args.dtype or cfg.dtype
    soap = Soap(cfg.species, r_cut=cfg.r_cut, n_max=cfg.n_max, l_max=cfg.l_max, sigma=cfg.sigma,
                average=cfg.average, dtype=dtype, alphas=alphas, betas=betas)
    dev = torch.device("cuda", 0)
    names = ("numbers", "positions", "cells", "pbc", "offsets")
    tensors = [torch.from_numpy(np.ascontiguousarray(getattr(batch, k))).to(dev) for k in names]
    out = torch.empty((soap.rows(batch), soap.feature_count),
                      dtype=torch.float32 if dtype == "float32" else torch.float64, device=dev)
    view = device_view(*(t.data_ptr() for t in tensors), batch.structures, batch.atoms)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for _ in range(args.repeats):
        soap.compute_device(view, out.data_ptr(), 0, stream)
    soap.check(0, stream)
    print(f"profile case: config {args.config}, {batch.structures} structures, {batch.atoms} atoms, "
          f"kernel {soap.kernel()}, {args.repeats} repeats")


if __name__ == "__main__":
    main()
