"""Fused tensor-parallel collective benchmark: ``torchrun --nproc-per-node N -m economize_b200.bench.tp_comm``.

Times on the device (the calls captured in one CUDA graph per path, replayed between CUDA events on every rank; the
max over ranks is reported) the row-parallel projection of a decode pass
followed by its all-reduce and RMSNorm, for the verification width of the benchmark tree (``--rows`` rows, default 61):

* ``fused``: ``FusedAllReduce.gemm_push`` (the tcgen05 GEMM stores its output tiles straight into every peer's
  slot over NVLink) + ``reduce_rmsnorm`` (sums the peers' slots, adds the residual, normalizes);
* ``nccl``: the same GEMM into a local tensor, ``torch.distributed.all_reduce`` (NCCL), then the RMSNorm kernel.

The roofline of one call is the slowest of its weight bytes at the measured HBM bandwidth, its FLOPs at the measured
bf16 peak and its NVLink bytes (each rank sends its ``M x H`` bf16 partial to every peer) at the measured 770 GB/s
per direction; the report gives each path's achieved fraction of it.
"""

from __future__ import annotations

import argparse
import json
import os

import torch

__all__ = ["main"]

NVLINK_GBS = 770.0  # measured peer copy bandwidth per direction on this pool's B200s


def main(argv: list[str] | None = None) -> None:
    import torch.distributed as dist

    from .. import ops
    from ..distributed import init_distributed
    from ..parallel.comm import FusedAllReduce
    from .cost_model import HARDWARE
    from .timing import max_over_ranks

    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--rows", type=int, default=61)
    p.add_argument("--hidden", type=int, default=4096)
    p.add_argument("--k", type=int, default=4096, help="full input width of the projection (split over ranks)")
    p.add_argument("--iters", type=int, default=200)
    p.add_argument("--warmup", type=int, default=20)
    a = p.parse_args(argv)
    tp = init_distributed("nccl", timeout_s=60)
    rank, world = tp.rank, tp.size
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(rank)
    k_local = a.k // world
    x = torch.randn(a.rows, k_local, device=dev, generator=g).bfloat16()
    w = (torch.randn(a.hidden, k_local, device=dev, generator=g) * 0.02).bfloat16()
    norm = torch.ones(a.hidden, device=dev).bfloat16()
    resid = torch.randn(a.rows, a.hidden, device=dev, generator=g).bfloat16()
    comm = FusedAllReduce(tp, a.hidden, max_tokens=max(256, a.rows))

    def fused():
        return comm.reduce_rmsnorm(comm.gemm_push(x, w), norm, 1e-5, resid)

    def nccl():
        y = ops.linear(x, w)
        dist.all_reduce(y, group=tp.group)
        return ops.rmsnorm(y, norm, 1e-5, resid)

    out = {}
    for name, fn in (("fused", fused), ("nccl", nccl)):
        for _ in range(a.warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier(group=tp.group)
        # device time only: the calls are captured once in a CUDA graph (both paths are capturable) and replayed
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(a.iters):
                fn()
        torch.cuda.synchronize()
        dist.barrier(group=tp.group)
        graph.replay()  # warm replay
        torch.cuda.synchronize()
        dist.barrier(group=tp.group)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        graph.replay()
        e.record()
        torch.cuda.synchronize()
        out[name] = max_over_ranks(s.elapsed_time(e) / a.iters, dev) * 1e3  # us
        del graph  # released before the process group is destroyed
        dist.barrier(group=tp.group)
    comm.check()
    hw = HARDWARE["b200"]  # the measured copy bandwidth and cuBLAS bf16 peak of this pool
    hbm_gbs, tflops = hw.hbm_gbs, hw.bf16_tflops
    weight_bytes = a.hidden * k_local * 2
    flops = 2 * a.rows * a.hidden * k_local
    link_bytes = (world - 1) * a.rows * a.hidden * 2
    t_hbm, t_flop, t_link = weight_bytes / hbm_gbs / 1e3, flops / tflops / 1e6, link_bytes / NVLINK_GBS / 1e3  # us
    roof = max(t_hbm, t_flop, t_link)
    if rank == 0:
        print(json.dumps({"op": "row_parallel_gemm_allreduce_rmsnorm", "ranks": world, "M": a.rows, "H": a.hidden,
                          "K": a.k, "fused_us": round(out["fused"], 2), "nccl_us": round(out["nccl"], 2),
                          "speedup": round(out["nccl"] / out["fused"], 3), "roofline_us": round(roof, 2),
                          "roofline_terms_us": {"hbm": round(t_hbm, 2), "tensor": round(t_flop, 3),
                                                "nvlink": round(t_link, 2)},
                          "fused_frac_of_roofline": round(roof / out["fused"], 3),
                          "nccl_frac_of_roofline": round(roof / out["nccl"], 3)}))
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
