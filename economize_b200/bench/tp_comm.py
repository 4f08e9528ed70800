"""Fused tensor-parallel collective benchmark: ``torchrun --nproc-per-node N -m economize_b200.bench.tp_comm``.

Times on the device (the calls captured in one CUDA graph per path, replayed between CUDA events on every rank; the
max over ranks is reported) one sublayer boundary of a decode pass at the verification width of the benchmark tree
(``--rows`` rows, default 61): a row-parallel projection (``--k`` input features split over the ranks, ``--hidden``
outputs), the sum over ranks, the residual add and RMSNorm, and the next column-parallel projection (``--n`` outputs
split over the ranks):

* ``sp``: the sequence-parallel fused path of :mod:`economize_b200.parallel.sp` -- GEMM -> reduce-scatter (output
  rows stored into their owner's slot over NVLink), reduce + residual + RMSNorm + all-gather push, all-gather ->
  GEMM (the next GEMM waits for every rank's rows);
* ``nccl``: the same GEMMs on local tensors around ``torch.distributed.all_reduce`` (NCCL) and the RMSNorm kernel;
* ``fused_ar``: the all-reduce formulation of :mod:`economize_b200.parallel.comm` (every rank's full partial pushed
  to every peer, summed and normalized on every rank) followed by the column GEMM.

The roofline of one boundary is the slowest of its weight bytes at the measured HBM bandwidth, its FLOPs at the
measured bf16 peak and the bytes a rank must send over NVLink (reduce-scatter + all-gather: ``2 (P - 1) / P`` times
the ``M x H`` bf16 rows) at the measured 770 GB/s per direction; the report gives each path's fraction of it.
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
    from ..parallel.sp import SequenceParallel
    from .cost_model import HARDWARE
    from .timing import max_over_ranks

    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--rows", type=int, default=61)
    p.add_argument("--hidden", type=int, default=4096)
    p.add_argument("--k", type=int, default=4096, help="full input width of the row-parallel projection")
    p.add_argument("--n", type=int, default=6144, help="full output width of the column-parallel projection")
    p.add_argument("--iters", type=int, default=200)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--breakdown", action="store_true", help="also print each kernel's device time per boundary "
                   "(CUPTI records of eager calls, rank 0)")
    a = p.parse_args(argv)
    tp = init_distributed("nccl", timeout_s=60)
    rank, world = tp.rank, tp.size
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(rank)
    k_local, n_local = a.k // world, a.n // world
    x = torch.randn(a.rows, k_local, device=dev, generator=g).bfloat16()
    w_row = (torch.randn(a.hidden, k_local, device=dev, generator=g) * 0.02).bfloat16()
    w_col = (torch.randn(n_local, a.hidden, device=dev, generator=g) * 0.02).bfloat16()
    norm = torch.ones(a.hidden, device=dev).bfloat16()
    resid = torch.randn(a.rows, a.hidden, device=dev, generator=torch.Generator(device=dev).manual_seed(9)).bfloat16()
    sp = SequenceParallel(tp, a.hidden, max_rows=max(256, a.rows))
    comm = FusedAllReduce(tp, a.hidden, max_tokens=max(256, a.rows))
    lo, n_own = sp.shard(a.rows)
    resid_own = resid[lo:lo + n_own].contiguous()

    def fused_sp():
        sp.rs_linear(x, w_row)
        sp.reduce_norm(resid_own, norm, 1e-5, a.rows)
        return sp.ag_linear(w_col, a.rows)

    def nccl():
        y = ops.linear(x, w_row)
        dist.all_reduce(y, group=tp.group)
        h, _ = ops.rmsnorm(y, norm, 1e-5, resid)
        return ops.linear(h, w_col)

    def fused_ar():
        h, _ = comm.reduce_rmsnorm(comm.gemm_push(x, w_row), norm, 1e-5, resid)
        return ops.linear(h, w_col)

    h_full = torch.randn(a.rows, a.hidden, device=dev, generator=g).bfloat16()

    def sp_no_col():  # the collective half alone: the all-gather round consumed by a copy instead of the GEMM
        sp.rs_linear(x, w_row)
        sp.reduce_norm(resid_own, norm, 1e-5, a.rows)
        return sp.fetch(a.rows, x)

    def gemms():  # the two projections alone, on local tensors
        ops.linear(x, w_row)
        return ops.linear(h_full, w_col)

    out = {}
    for name, fn in (("sp", fused_sp), ("nccl", nccl), ("fused_ar", fused_ar), ("sp_no_col_gemm", sp_no_col),
                     ("gemms_only", gemms)):
        for _ in range(a.warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier(group=tp.group)
        # device time only: the calls are captured once in a CUDA graph (every path is capturable) and replayed
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
    if a.breakdown:
        from torch.profiler import ProfilerActivity, profile

        for name, fn in (("sp", fused_sp), ("nccl", nccl)):
            torch.cuda.synchronize()
            dist.barrier(group=tp.group)
            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                for _ in range(20):
                    fn()
                torch.cuda.synchronize()
            dist.barrier(group=tp.group)
            per: dict[str, float] = {}
            for ev in prof.events():
                if ev.device_type == torch.autograd.DeviceType.CUDA:
                    per[ev.name[:60]] = per.get(ev.name[:60], 0.0) + ev.device_time_total / 20
            if rank == 0:
                print(json.dumps({"breakdown": name, "us_per_boundary": {k: round(v, 2) for k, v in
                                                                         sorted(per.items(), key=lambda kv: -kv[1])}}))
    sp.check()
    comm.check()
    hw = HARDWARE["b200"]  # the measured copy bandwidth and cuBLAS bf16 peak of this pool
    hbm_gbs, tflops = hw.hbm_gbs, hw.bf16_tflops
    weight_bytes = (a.hidden * k_local + n_local * a.hidden) * 2
    flops = 2 * a.rows * (a.hidden * k_local + n_local * a.hidden)
    link_bytes = 2 * (world - 1) / world * a.rows * a.hidden * 2
    t_hbm, t_flop, t_link = weight_bytes / hbm_gbs / 1e3, flops / tflops / 1e6, link_bytes / NVLINK_GBS / 1e3  # us
    roof = max(t_hbm, t_flop, t_link)
    if rank == 0:
        print(json.dumps({"op": "row_gemm_rs_norm_ag_col_gemm", "ranks": world, "M": a.rows, "H": a.hidden,
                          "K": a.k, "N": a.n, "sp_us": round(out["sp"], 2), "nccl_us": round(out["nccl"], 2),
                          "fused_allreduce_us": round(out["fused_ar"], 2),
                          "sp_without_column_gemm_us": round(out["sp_no_col_gemm"], 2),
                          "two_gemms_alone_us": round(out["gemms_only"], 2),
                          "sp_vs_nccl": round(out["nccl"] / out["sp"], 3), "roofline_us": round(roof, 2),
                          "roofline_terms_us": {"hbm": round(t_hbm, 2), "tensor": round(t_flop, 3),
                                                "nvlink": round(t_link, 2)},
                          "sp_frac_of_roofline": round(roof / out["sp"], 3),
                          "nccl_frac_of_roofline": round(roof / out["nccl"], 3)}))
    sp.close()
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
