"""Kernel micro-benchmarks: ``python -m economize_b200.bench.kernels <op> [options]``.

Each op times the engine's kernel (and, where one exists, the library baseline on the same shapes) with
:func:`~economize_b200.bench.timing.time_call` (CUDA events per call, L2 flushed before every call, warm-up first)
and prints one JSON line with the median time, the algorithmic bytes/FLOPs and the fraction of the measured
peaks. Ops:

* ``gemm``       bf16 ``x[M, K] @ w[N, K]^T`` (tcgen05 swap-AB GEMM vs cuBLAS through torch.matmul); calls on
  rotating weight copies (more than 2x L2 in total) are captured in one CUDA graph, so the per-call time excludes
  launch overhead and reads the weights from HBM
* ``gemm_sweep`` every GEMM variant of the engine and cuBLAS at the decode shapes of Llama-3.1-8B (``--ms`` token
  counts); one JSON line per shape
* ``gemm_wq``    weight-only int2 / int4 / int8 / fp8 / mxfp4 / nvfp4 GEMM (``--fmt``), vs the bf16 kernel on the
  same shape
* ``hadamard``   SwiGLU with the online Hadamard rotation fused (block ``--group``, width ``--n``) vs the plain
  SwiGLU kernel on the same input
* ``attention``  tree-masked decode attention over a bf16 slot cache (``--tree`` new tokens per row)
* ``layer``      one Llama-3.1-8B decoder layer's projections as a CUDA graph (``--tp`` shard), ours vs cuBLAS
* ``teal``       activation-sparse GEMV (``colsparse_linear`` over a transposed weight) at ``--sparsity`` of the
  input entries dropped, vs the dense tcgen05 GEMM on the same shape; bytes are the weight rows actually needed
* ``glu``        CATS's gated rows (``glu_rows``: up rows of the channels with ``|silu(gate)| > t``, ``--n`` = FFN
  width, ``--k`` = hidden) at ``--sparsity``, vs the dense up projection GEMM

``--once`` runs a single call without timing (the case a profiler captures).
"""

from __future__ import annotations

import argparse
import json
import sys

import torch

from .cost_model import HARDWARE
from .timing import L2_BYTES, time_call, time_graph

__all__ = ["main"]


def _peaks() -> tuple[float, float]:
    hw = HARDWARE["b200"]
    return hw.hbm_gbs, hw.bf16_tflops


def _report(name: str, shape: dict, ms: float, nbytes: float, flops: float, baseline_ms: float | None = None):
    hbm, tflops = _peaks()
    out = {"op": name, **shape, "us": round(ms * 1e3, 2), "GB_s": round(nbytes / ms / 1e6, 1),
           "TFLOP_s": round(flops / ms / 1e9, 1), "hbm_frac_of_measured": round(nbytes / ms / 1e6 / hbm, 3),
           "tensor_frac_of_measured": round(flops / ms / 1e9 / tflops, 3)}
    if baseline_ms is not None:
        out["baseline_us"] = round(baseline_ms * 1e3, 2)
        out["speedup"] = round(baseline_ms / ms, 3)
    print(json.dumps(out))
    sys.stdout.flush()


def _copies(nbytes: int) -> int:
    """Distinct weight copies so that one pass over all of them streams at least 2x L2 from HBM."""
    return max(2, -(-2 * L2_BYTES // max(nbytes, 1)))


def bench_gemm(a) -> None:
    from .. import ops

    dev = torch.device("cuda")
    x = torch.randn(a.m, a.k, device=dev).bfloat16()
    n_copies = 1 if a.once else _copies(2 * a.n * a.k)
    ws = [(torch.randn(a.n, a.k, device=dev) * 0.02).bfloat16() for _ in range(n_copies)]
    if a.once:
        ops.linear(x, ws[0])
        torch.cuda.synchronize()
        return
    # --parts: the split-K kernel whose fp32 partials a fused consumer (norm, SwiGLU, RoPE) reduces, as decode runs it
    fn = (lambda w: ops.linear_parts(x, w)) if a.parts else (lambda w: ops.linear(x, w))
    ours = time_graph([lambda w=w: fn(w) for w in ws], a.iters, a.warmup)
    base = time_graph([lambda w=w: torch.matmul(x, w.t()) for w in ws], a.iters, a.warmup)
    nbytes = 2 * (a.m * a.k + a.n * a.k + a.m * a.n)
    _report("gemm_parts" if a.parts else "gemm", {"M": a.m, "N": a.n, "K": a.k, "copies": n_copies}, ours, nbytes,
            2 * a.m * a.n * a.k, base)


def bench_gemm_sweep(a) -> None:
    """Every GEMM variant (``linear_variant`` modes) and cuBLAS at the decode shapes of Llama-3.1-8B: one JSON line
    per (M, N, K) with the microseconds of each (CUDA graph over rotating weight copies, weights from HBM)."""
    from .. import ops

    ext = ops.require()
    dev = torch.device("cuda")
    hbm, _ = _peaks()
    shapes = [(6144, 4096), (4096, 4096), (28672, 4096), (4096, 14336), (128256, 4096)]
    modes = {"cluster": 1, "splitk_lastcta": 2, "stream_k": 3, "parts_2cta": 4, "splitk_2cta_lastcta": 6}
    for m in a.ms:
        for n, k in shapes:
            x = torch.randn(m, k, device=dev).bfloat16()
            ws = [(torch.randn(n, k, device=dev) * 0.02).bfloat16() for _ in range(_copies(2 * n * k))]
            row = {"op": "gemm_sweep", "M": m, "N": n, "K": k}
            nbytes = 2 * (m * k + n * k + m * n)
            for name, mode in modes.items():
                try:
                    t = time_graph([lambda w=w, mode=mode: ext.linear_variant(x, w, mode, 0) for w in ws], a.iters,
                                   a.warmup)
                    row[name] = round(t * 1e3, 2)
                except RuntimeError as err:
                    row[name] = f"n/a ({str(err)[:40]})"
            row["default"] = round(time_graph([lambda w=w: ops.linear(x, w) for w in ws], a.iters, a.warmup) * 1e3, 2)
            row["parts_default"] = round(time_graph([lambda w=w: ops.linear_parts(x, w) for w in ws], a.iters,
                                                    a.warmup) * 1e3, 2)
            row["cublas"] = round(time_graph([lambda w=w: torch.matmul(x, w.t()) for w in ws], a.iters,
                                             a.warmup) * 1e3, 2)
            best = min(v for v in row.values() if isinstance(v, float))
            row["roofline_us"] = round(nbytes / hbm / 1e3, 2)
            row["best_frac_of_measured_hbm"] = round(nbytes / hbm / 1e3 / best, 3)
            print(json.dumps(row))
            sys.stdout.flush()
            del ws


def bench_gemm_wq(a) -> None:
    from .. import ops
    from ..techniques.quant import rtn

    dev = torch.device("cuda")
    x = torch.randn(a.m, a.k, device=dev).bfloat16()
    w = torch.randn(a.n, a.k, device=dev) * 0.02
    qw0 = rtn(w, a.fmt, a.group, a.fmt not in ("int2", "int4"))
    if a.once:
        ops.linear(x, qw0)
        torch.cuda.synchronize()
        return
    qws = [qw0] + [rtn(w, a.fmt, a.group, a.fmt not in ("int2", "int4")) for _ in range(_copies(qw0.nbytes()) - 1)]
    wbs = [w.bfloat16() for _ in range(_copies(2 * a.n * a.k))]
    ours = time_graph([lambda q=q: ops.linear(x, q) for q in qws], a.iters, a.warmup)
    bf16 = time_graph([lambda wb=wb: ops.linear(x, wb) for wb in wbs], a.iters, a.warmup)
    nbytes = qw0.nbytes() + 2 * (a.m * a.k + a.m * a.n)
    _report(f"gemm_{a.fmt}", {"M": a.m, "N": a.n, "K": a.k, "group": a.group}, ours, nbytes, 2 * a.m * a.n * a.k,
            bf16)


def bench_attention(a) -> None:
    from .. import ops
    from ..decoding.tree import ancestor_bits

    dev = torch.device("cuda")
    B, T, H, Hkv, D = a.batch, a.tree, 32 // a.tp, 8 // a.tp, 128
    S = ((a.ctx + T + 127) // 128) * 128
    k = torch.randn(B, Hkv, S, D, device=dev).bfloat16()
    v = torch.randn(B, Hkv, S, D, device=dev).bfloat16()
    q = torch.randn(B, T, H, D, device=dev).bfloat16()
    kv_len = torch.full((B,), a.ctx, dtype=torch.int32, device=dev)
    n_new = torch.full((B,), T, dtype=torch.int32, device=dev)
    parents = torch.arange(-1, T - 1, device=dev)[None].expand(B, T)  # a chain (worst case: full depth)
    mask = ancestor_bits(parents.contiguous(), T) if T > 1 else None
    tail = a.tail if T <= 64 else 0
    if a.once:
        ops.attention(q, k, v, kv_len, n_new, mask, tail=tail)
        torch.cuda.synchronize()
        return
    if a.trace:
        _attention_timeline(q, k, v, kv_len, n_new, mask, a)
        return
    ours = time_graph([lambda: ops.attention(q, k, v, kv_len, n_new, mask, tail=tail)] * 8, a.iters, a.warmup)
    nbytes = 2 * (2 * B * Hkv * (a.ctx + T) * D + 2 * B * T * H * D)
    flops = 4 * B * T * H * (a.ctx + T) * D
    _report("attention", {"B": B, "T": T, "H": H, "Hkv": Hkv, "ctx": a.ctx, "tail": tail}, ours, nbytes, flops)


def _steady_phases(st, med) -> dict:
    """Phase times in SM cycles of the pipelined walk's third chunk (stamps 8-15: loop top, scores ready, loads
    issued, row maxima shared, previous P . V done, P stored, P visible to the MMA issuer, P . V issued)."""
    fine = st[st[:, 15] != 0]
    if fine.shape[0] == 0:
        return {}
    names = ["wait_s", "issue", "max", "wait_pv", "p_store", "sync", "pv_issue"]
    out = {f"c2_{n}_cyc": int(med(fine[:, 9 + j] - fine[:, 8 + j]) * 1e3) for j, n in enumerate(names)}
    out["c2_total_cyc"] = int(med(fine[:, 15] - fine[:, 8]) * 1e3)
    return out


def _attention_timeline(q, k, v, kv_len, n_new, mask, a) -> None:
    """Per-CTA phase times of the attention kernel from its global-timer stamps (start, TMEM + Q staged, first K/V
    chunk landed, first S MMA done, first softmax done, first PV MMA done, chunk loop done, end): medians over the
    CTAs, the number of CTAs resident at once, and the kernel's span from the first start to the last end."""
    from .. import ops

    C = ops.require()
    B, T, H, D = q.shape
    Hkv, S = k.shape[1], k.shape[2]
    most = B * Hkv * -(-T * (H // Hkv) // 128) * (S // 128)
    trace = torch.zeros(most * 16, dtype=torch.int64, device=q.device)
    for _ in range(a.warmup):
        ops.attention(q, k, v, kv_len, n_new, mask)
    C.attention(q, k, v, kv_len, n_new, mask, D ** -0.5, 0, trace)
    torch.cuda.synchronize()
    st = trace.view(-1, 16).cpu()
    st = st[st[:, 0] != 0].double()
    if st.shape[0] == 0:
        print(json.dumps({"op": "attention_timeline", "error": "no stamps"}))
        return
    span_us = float((st[:, 7].max() - st[:, 0].min()) / 1e3)
    med = lambda x: round(float(x.median()) / 1e3, 3)  # noqa: E731
    sms = torch.cuda.get_device_properties(q.device).multi_processor_count
    _, splits, chunks = C.attention_plan(B, T, H, Hkv, S, sms)
    starts = st[:, 0].sort().values
    ends = st[:, 7].sort().values
    resident = int(max(((starts <= t0) & (ends > t0)).sum() for t0 in starts[:: max(1, len(starts) // 64)]))
    print(json.dumps({"op": "attention_timeline", "T": T, "ctx": a.ctx, "ctas": int(st.shape[0]),
                      "resident_max": resident, "span_us": round(span_us, 2),
                      "setup_us": med(st[:, 1] - st[:, 0]), "first_kv_us": med(st[:, 2] - st[:, 0]),
                      "s_mma_us": med(st[:, 3] - st[:, 2]), "softmax_us": med(st[:, 4] - st[:, 3]),
                      "pv_us": med(st[:, 5] - st[:, 4]), "loop_us": med(st[:, 6] - st[:, 2]),
                      "epilogue_us": med(st[:, 7] - st[:, 6]), "cta_us": med(st[:, 7] - st[:, 0]),
                      **_steady_phases(st, med),
                      "splits": int(splits), "chunks_per_split": int(chunks)}))


def bench_layer(a) -> None:
    from .. import ops

    dev = torch.device("cuda")
    tp = a.tp
    H, F, Q, KV = 4096, 14336 // tp, 4096 // tp, 1024 // tp
    n_layers = 8

    def mk(n, k):
        return (torch.randn(n, k, device=dev) * 0.02).bfloat16()

    layers = [dict(qkv=mk(Q + 2 * KV, H), o=mk(H, Q), gu=mk(2 * F, H), d=mk(H, F)) for _ in range(n_layers)]
    x = torch.randn(a.m, H, device=dev).bfloat16()

    def chain(lin):
        h = x
        for L in layers:
            q = lin(h, L["qkv"])
            o = lin(q[:, :Q].contiguous(), L["o"])
            g = lin(o, L["gu"])
            h = lin(g[:, :F].contiguous(), L["d"])
        return h

    res = {}
    for name, lin in (("ours", ops.linear), ("cublas", lambda t, w: torch.matmul(t, w.t()))):
        chain(lin)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            chain(lin)
        res[name] = time_call(g.replay, a.iters, a.warmup, flush=False).median_ms / n_layers
        del g
    nbytes = sum(v.numel() * 2 for v in layers[0].values())
    flops = 2 * a.m * sum(v.numel() for v in layers[0].values())
    _report("layer_projections", {"M": a.m, "tp": tp}, res["ours"], nbytes, flops, res["cublas"])


def bench_teal(a) -> None:
    from .. import ops
    from ..ops._ext import require

    dev = torch.device("cuda")
    C = require()
    x = torch.randn(a.m, a.k, device=dev).bfloat16()
    t = torch.quantile(x.float().abs().flatten()[:1 << 20], a.sparsity).reshape(()) if a.sparsity > 0 else \
        torch.zeros((), device=dev)
    n_copies = 1 if a.once else _copies(2 * a.n * a.k)
    ws = [(torch.randn(a.n, a.k, device=dev) * 0.02).bfloat16() for _ in range(n_copies)]
    wts = [w.t().contiguous() for w in ws]
    if a.once:
        C.colsparse_linear(x, wts[0], t)
        torch.cuda.synchronize()
        return
    ours = time_graph([lambda wt=wt: C.colsparse_linear(x, wt, t) for wt in wts], a.iters, a.warmup)
    dense = time_graph([lambda w=w: ops.linear(x, w) for w in ws], a.iters, a.warmup)
    kept = float((x.abs() > t.bfloat16()).any(0).float().mean())
    nbytes = 2 * (a.m * a.k + kept * a.n * a.k + a.m * a.n)
    _report("teal_gemv", {"M": a.m, "N": a.n, "K": a.k, "sparsity": a.sparsity, "rows_kept": round(kept, 3)}, ours,
            nbytes, 2 * a.m * a.n * a.k * kept, dense)


def bench_topk(a) -> None:
    """Fused log-softmax + top-k over ``[m, n]`` fp32 logits (draft-tree expansion) vs torch's three kernels."""
    from .. import ops

    dev = torch.device("cuda")
    xs = [torch.randn(a.m, a.n, device=dev) for _ in range(_copies(4 * a.m * a.n))]
    d2t = torch.randint(0, 100000, (a.n,), device=dev)  # a draft-to-target id map, as EAGLE-3 heads use
    if a.once:
        ops.topk_logp(xs[0], a.topk, -1e4, d2t)
        torch.cuda.synchronize()
        return
    ours = time_graph([lambda x=x: ops.topk_logp(x, a.topk, -1e4, d2t) for x in xs], a.iters, a.warmup)
    base = time_graph([lambda x=x: torch.log_softmax(x, -1).topk(a.topk, -1) for x in xs], a.iters, a.warmup)
    _report("topk_logp", {"rows": a.m, "V": a.n, "k": a.topk}, ours, 4 * a.m * a.n, 0, base)


def bench_glu(a) -> None:
    from .. import ops
    from ..ops._ext import require

    dev = torch.device("cuda")
    C = require()
    F_, H = a.n, a.k
    x = torch.randn(a.m, H, device=dev).bfloat16()
    n_copies = 1 if a.once else _copies(4 * F_ * H)
    ws = [(torch.randn(2 * F_, H, device=dev) * 0.02).bfloat16() for _ in range(n_copies)]
    gates = [ops.linear(x, w[:F_]) for w in ws]
    s = torch.nn.functional.silu(gates[0].float()).abs().flatten()
    t = torch.quantile(s, a.sparsity).reshape(()) if a.sparsity > 0 else torch.zeros((), device=dev)
    if a.once:
        C.glu_rows(x, ws[0], gates[0], None, t)
        torch.cuda.synchronize()
        return
    ours = time_graph([lambda w=w, g=g: C.glu_rows(x, w, g, None, t) for w, g in zip(ws, gates)], a.iters, a.warmup)
    ups = [w[F_:] for w in ws]
    dense = time_graph([lambda u=u: ops.linear(x, u) for u in ups], a.iters, a.warmup)
    kept = float((torch.nn.functional.silu(gates[0].float()).abs() > t).any(0).float().mean())
    nbytes = 2 * (a.m * H + kept * F_ * H + 2 * a.m * F_)
    _report("cats_glu_rows", {"M": a.m, "F": F_, "H": H, "sparsity": a.sparsity, "rows_kept": round(kept, 3)}, ours,
            nbytes, 2 * a.m * F_ * H * kept, dense)


def bench_hadamard(a) -> None:
    """The gated activation with the online Hadamard rotation fused (``glu_hadamard``) against the plain gated
    activation (``silu_mul``) of the same ``[M, 2F]`` input, inputs rotated over copies larger than L2."""
    from ..ops._ext import require

    dev = torch.device("cuda")
    C = require()
    F_ = a.n
    block = a.group if a.group >= 8 else 2048
    n_copies = 1 if a.once else _copies(4 * a.m * F_)
    gus = [torch.randn(a.m, 2 * F_, device=dev).bfloat16() for _ in range(n_copies)]
    if a.once:
        C.glu_hadamard(gus[0], 0, 7.0, block)
        torch.cuda.synchronize()
        return
    fused = time_graph([lambda g=g: C.glu_hadamard(g, 0, 7.0, block) for g in gus], a.iters, a.warmup)
    plain = time_graph([lambda g=g: C.silu_mul(g) for g in gus], a.iters, a.warmup)
    _report("glu_hadamard", {"M": a.m, "F": F_, "block": block}, fused, 2 * (2 * a.m * F_ + a.m * F_),
            a.m * F_ * (block.bit_length() - 1), plain)


def main(argv: list[str] | None = None) -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("op", choices=["gemm", "gemm_sweep", "gemm_wq", "attention", "layer", "teal", "glu", "topk",
                                  "hadamard"])
    p.add_argument("--ms", type=int, nargs="+", default=[1, 8, 61, 488], help="gemm_sweep: token counts")
    p.add_argument("--topk", type=int, default=10)
    p.add_argument("--m", type=int, default=61)
    p.add_argument("--n", type=int, default=6144)
    p.add_argument("--k", type=int, default=4096)
    p.add_argument("--parts", action="store_true", help="gemm: time the split-K partials kernel of decode")
    p.add_argument("--fmt", default="int4", choices=["int2", "int4", "int8", "fp8", "mxfp4", "nvfp4"])
    p.add_argument("--group", type=int, default=128)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--tree", type=int, default=61)
    p.add_argument("--ctx", type=int, default=768)
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--sparsity", type=float, default=0.5)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--once", action="store_true", help="one untimed call (for profiler captures)")
    p.add_argument("--tail", type=int, default=0, help="attention: exact-tail width (decode passes use 16)")
    p.add_argument("--trace", action="store_true", help="attention: per-CTA phase timeline from the kernel's stamps")
    a = p.parse_args(argv)
    {"gemm": bench_gemm, "gemm_sweep": bench_gemm_sweep, "gemm_wq": bench_gemm_wq, "attention": bench_attention, "layer": bench_layer,
     "teal": bench_teal, "glu": bench_glu, "topk": bench_topk, "hadamard": bench_hadamard}[a.op](a)


if __name__ == "__main__":
    main()
