"""Quantization methods: round to nearest, GPTQ and AWQ, producing the packed kernel layout.

* RTN: min-max (asymmetric) or abs-max (symmetric) grids per (output row, group).
* GPTQ (Frantar et al., 2022, "GPTQ: Accurate Post-Training Quantization for Generative Pre-trained Transformers"):
  columns are quantized in order while the rounding error of each column is spread over the not-yet-quantized
  columns through the upper Cholesky factor of the inverse damped Hessian ``H = 2 X^T X / n``, in lazy blocks.
  Group grids are fitted when the first column of a group is reached (on the already-updated weights), or on the
  original weights with ``act_order`` (static groups). Economize's implementation: ``techniques/quant/gptq.py``.
* AWQ (Lin et al., 2023, "AWQ: Activation-aware Weight Quantization"): per input channel scales
  ``s = mean|x|^a`` (normalised) for the exponent ``a`` on a grid that minimises the output error of the quantized
  map, folded exactly into the preceding RMSNorm weight (or the producing projection's rows), followed by a search
  of per-group clipping ratios. Economize's implementation: ``techniques/quant/awq.py``.

Calibration runs the engine model once per layer chunk with an observer that receives the input of every projection
(economize's layer-wise calibration engine, ``core/calibration.py``); statistics are taken from the
full-precision model (all layers observed in the same passes, not re-run after each layer is quantized).
"""

from __future__ import annotations

import math
from collections.abc import Callable, Sequence

import torch

from ...errors import ConfigError
from ...ops.quant import FP4_GROUP, QWeight, e2m1_round, pack

__all__ = ["Grid", "awq_search", "collect", "fit_grid", "gptq", "quantize_codes", "rtn"]

FP8_MAX = 448.0
#: largest code of the zero-point integer formats
_INT_TOP = {"int2": 3.0, "int3": 7.0, "int4": 15.0}


class Grid:
    """Per (row, group) scales (and int4 zero points) of one weight matrix.

    ``scale [N, G]`` fp32 holding bf16-representable values, ``zero [N, G]`` fp32 integer zero points (int4) or
    ``None``.
    """

    def __init__(self, scale: torch.Tensor, zero: torch.Tensor | None) -> None:
        self.scale, self.zero = scale, zero


def _mx_scale(amax: torch.Tensor) -> torch.Tensor:
    """MXFP4 group scale: ``2^(e - 2)`` with ``e`` the exponent of ``amax`` rounded to a power of two (up when its
    mantissa is at least 1.75, so the group maximum lands at 4..7 units instead of clipping at 6)."""
    e = torch.floor(torch.log2(amax.clamp(min=2.0 ** -120)))
    e = torch.where(amax / torch.exp2(e) >= 1.75, e + 1, e)
    return torch.where(amax > 0, torch.exp2(e - 2), torch.ones_like(amax))


def nvfp4_global_scale(amax: float) -> float:
    """NVFP4 global scale: the power of two at or below ``448 * 6 / amax`` (so the largest group scale fits e4m3 and
    every effective scale ``s8 / global`` is exact in bf16)."""
    if amax <= 0:
        return 1.0
    return float(2.0 ** math.floor(math.log2(448.0 * 6.0 / amax)))


def _fp4_grid(w: torch.Tensor, fmt: str, clip, tensor_amax: float | None) -> Grid:
    amax = w.abs().amax(-1) * clip
    if fmt == "mxfp4":
        return Grid(_mx_scale(amax), None)
    glob = nvfp4_global_scale(float(w.abs().max()) if tensor_amax is None else float(tensor_amax))
    s8 = (amax / 6.0 * glob).clamp(2.0 ** -9, 448.0).to(torch.float8_e4m3fn).float()
    return Grid(s8.clamp(min=2.0 ** -9) / glob, None)


def fit_grid(w: torch.Tensor, fmt: str, symmetric: bool, clip: torch.Tensor | float = 1.0,
             tensor_amax: float | None = None) -> Grid:
    """Grid of ``w [N, G, g]`` (groups along the last axis); ``clip`` shrinks the range (AWQ's clipping).
    ``tensor_amax``: the whole weight's absolute maximum, for NVFP4's global scale when ``w`` is part of it."""
    if fmt in FP4_GROUP:
        return _fp4_grid(w, fmt, clip, tensor_amax)
    top = _INT_TOP.get(fmt)
    if top is not None and not symmetric:
        hi = (w.amax(-1) * clip).clamp(min=0)
        lo = (w.amin(-1) * clip).clamp(max=0)
        same = (hi - lo) == 0
        lo, hi = torch.where(same, -torch.ones_like(lo), lo), torch.where(same, torch.ones_like(hi), hi)
        scale = ((hi - lo) / top).to(torch.bfloat16).float()
        zero = torch.round(-lo / scale).clamp(0, top)
        return Grid(scale, zero)
    amax = w.abs().amax(-1) * clip
    levels = {"int2": 1.0, "int3": 3.0, "int4": 7.0, "int8": 127.0, "fp8": FP8_MAX}[fmt]
    scale = (amax / levels).to(torch.bfloat16).float()
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    return Grid(scale, torch.full_like(scale, (top + 1) / 2) if top is not None else None)


def quantize_codes(w: torch.Tensor, grid: Grid, fmt: str) -> tuple[torch.Tensor, torch.Tensor]:
    """Codes and dequantized values (bf16-rounded, fp32) of ``w [N, G, g]`` on ``grid``."""
    s = grid.scale[..., None]
    if fmt in _INT_TOP:
        z = grid.zero[..., None]
        q = torch.clamp(torch.round(w / s) + z, 0, _INT_TOP[fmt])
        return q, ((q - z) * s).to(torch.bfloat16).float()
    if fmt == "int8":
        q = torch.clamp(torch.round(w / s), -128, 127)
        return q, (q * s).to(torch.bfloat16).float()
    if fmt in FP4_GROUP:
        q = e2m1_round(w / s)
        return q, (q * s).to(torch.bfloat16).float()
    q = (w / s).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).float()
    return q, (q * s).to(torch.bfloat16).float()


def _qweight(codes: torch.Tensor, grid: Grid, fmt: str, group: int, dtype: torch.dtype) -> QWeight:
    n = codes.shape[0]
    codes = codes.reshape(n, -1)
    packed = pack(codes.to(torch.float8_e4m3fn) if fmt == "fp8" else codes if fmt in FP4_GROUP
                  else codes.to(torch.int64), fmt)
    scales = grid.scale.t().contiguous().to(torch.bfloat16)
    zeros = (grid.zero.t() + 128.0).contiguous().to(torch.bfloat16) if fmt in _INT_TOP else None
    return QWeight(packed, scales, zeros, fmt, group, dtype)


def _groups(w: torch.Tensor, group: int) -> torch.Tensor:
    n, k = w.shape
    if k % group:
        raise ConfigError(f"group size {group} does not divide the input width {k}")
    return w.reshape(n, k // group, group)


def rtn(weight: torch.Tensor, fmt: str, group: int | None, symmetric: bool,
        clip: torch.Tensor | float = 1.0) -> QWeight:
    """Round-to-nearest quantization of ``weight [N, K]`` (FP4 formats use their own group of 32 or 16)."""
    g = FP4_GROUP.get(fmt) or group or weight.shape[1]
    w = _groups(weight.float(), g)
    grid = fit_grid(w, fmt, symmetric, clip)
    codes, _ = quantize_codes(w, grid, fmt)
    return _qweight(codes, grid, fmt, g, weight.dtype)


@torch.no_grad()
def gptq(weight: torch.Tensor, hessian: torch.Tensor, fmt: str, group: int | None, symmetric: bool,
         blocksize: int = 128, percdamp: float = 0.01, act_order: bool = False) -> QWeight:
    """GPTQ of ``weight [N, K]`` given ``hessian [K, K]`` (``X^T X`` summed over calibration rows)."""
    W = weight.float().clone()
    n, k = W.shape
    g = FP4_GROUP.get(fmt) or group or k
    tensor_amax = float(W.abs().max())
    H = hessian.float().clone()
    dead = torch.diag(H) == 0
    H[dead, dead] = 1.0
    W[:, dead] = 0.0
    static = None
    if act_order:  # fit every group on the original contiguous columns, then visit columns by saliency
        static = fit_grid(_groups(W, g), fmt, symmetric, tensor_amax=tensor_amax)
        perm = torch.argsort(torch.diag(H), descending=True)
        W, H = W[:, perm], H[perm][:, perm]
        inv_perm = torch.argsort(perm)
    damp = percdamp * torch.mean(torch.diag(H))
    H += damp * torch.eye(k, device=H.device, dtype=H.dtype)
    L = torch.linalg.cholesky(H)
    Hinv = torch.linalg.cholesky(torch.cholesky_inverse(L), upper=True)
    codes = torch.zeros_like(W)
    scale = torch.zeros(n, k // g, device=W.device)
    zero = torch.zeros(n, k // g, device=W.device) if fmt in _INT_TOP else None
    cur: Grid | None = None
    for i1 in range(0, k, blocksize):
        i2 = min(i1 + blocksize, k)
        W1 = W[:, i1:i2].clone()
        err1 = torch.zeros_like(W1)
        Hinv1 = Hinv[i1:i2, i1:i2]
        for i in range(i2 - i1):
            col = i1 + i
            orig = int(perm[col]) if act_order else col
            grp = orig // g
            if act_order:
                cur = Grid(static.scale[:, grp:grp + 1], None if static.zero is None else static.zero[:, grp:grp + 1])
            elif col % g == 0:
                span = W1[:, i:i + g] if i + g <= i2 - i1 else torch.cat([W1[:, i:], W[:, i2:col + g]], 1)
                cur = fit_grid(span[:, None, :], fmt, symmetric, tensor_amax=tensor_amax)
                scale[:, grp] = cur.scale[:, 0]
                if zero is not None:
                    zero[:, grp] = cur.zero[:, 0]
            w = W1[:, i]
            q, dq = quantize_codes(w[:, None, None], cur, fmt)
            codes[:, col] = q[:, 0, 0]
            e = (w - dq[:, 0, 0]) / Hinv1[i, i]
            W1[:, i:] -= e[:, None] * Hinv1[i, i:][None, :]
            err1[:, i] = e
        W[:, i2:] -= err1 @ Hinv[i1:i2, i2:]
    if act_order:
        codes = codes[:, inv_perm]
        grid = static
    else:
        grid = Grid(scale, zero)
    return _qweight(codes, grid, fmt, g, weight.dtype)


# ---- calibration ----------------------------------------------------------------------------------------------
class _Stats:
    """Per-projection input statistics: ``X^T X`` (GPTQ), mean |x| per channel and a row sample (AWQ)."""

    def __init__(self, hessian: bool, keep_rows: int) -> None:
        self.hessian_on, self.keep_rows = hessian, keep_rows
        self.h: torch.Tensor | None = None
        self.abs_sum: torch.Tensor | None = None
        self.rows: list[torch.Tensor] = []
        self.kept = 0
        self.n = 0

    def add(self, x: torch.Tensor) -> None:
        x = x.reshape(-1, x.shape[-1]).float()
        if self.hessian_on:
            self.h = x.t() @ x if self.h is None else self.h.add_(x.t() @ x)
        self.abs_sum = x.abs().sum(0) if self.abs_sum is None else self.abs_sum.add_(x.abs().sum(0))
        if self.kept < self.keep_rows:
            take = x[: self.keep_rows - self.kept]
            self.rows.append(take.clone())
            self.kept += take.shape[0]
        self.n += x.shape[0]

    @property
    def hessian(self) -> torch.Tensor:
        return self.h * (2.0 / max(self.n, 1))

    @property
    def abs_mean(self) -> torch.Tensor:
        return self.abs_sum / max(self.n, 1)

    @property
    def sample(self) -> torch.Tensor:
        return torch.cat(self.rows, 0)


@torch.no_grad()
def collect(model, batches: Sequence[torch.Tensor], wanted: dict[int, Sequence[str]], hessian: bool,
            keep_rows: int) -> dict[tuple[int, str], _Stats]:
    """Input statistics of the projections ``wanted {layer: names}`` over calibration token batches ``[B, L]``."""
    from ...runtime.cache import StepBatch

    stats = {(i, n): _Stats(hessian, keep_rows) for i, names in wanted.items() for n in names}

    def observer(layer: int, name: str, x: torch.Tensor) -> None:
        s = stats.get((layer, name))
        if s is not None:
            s.add(x)

    model.observer = observer
    try:
        last = max(wanted) if wanted else -1
        for tokens in batches:
            tokens = tokens.to(model.device)
            if tokens.dim() == 1:
                tokens = tokens[None]
            b, length = tokens.shape
            cache = model.new_cache(b, ((length + 127) // 128) * 128)
            lengths = torch.full((b,), length, dtype=torch.int32, device=model.device)
            model.forward_step(tokens, StepBatch.prefill(lengths, length), cache, layers=range(last + 1))
    finally:
        model.observer = None
    return stats


# ---- AWQ -----------------------------------------------------------------------------------------------------
def _awq_loss(x: torch.Tensor, w: torch.Tensor, s: torch.Tensor, fmt: str, group: int, symmetric: bool) -> float:
    """Output error of quantizing ``w * s`` and feeding ``x / s``."""
    group = FP4_GROUP.get(fmt, group)
    ws = w * s[None, :]
    wq = _groups(ws, group)
    grid = fit_grid(wq, fmt, symmetric)
    _, dq = quantize_codes(wq, grid, fmt)
    y_ref = x @ w.t()
    y_q = (x / s[None, :]) @ dq.reshape_as(w).t()
    return float((y_ref - y_q).pow(2).mean())


@torch.no_grad()
def awq_search(weights: Sequence[torch.Tensor], stats: _Stats, fmt: str, group: int, symmetric: bool,
               grid_points: int) -> torch.Tensor:
    """The best input-channel scale of the maps ``weights`` (which share the input) over the exponent grid."""
    x = stats.sample
    w = torch.cat([wt.float() for wt in weights], 0)
    mean = stats.abs_mean.clamp(min=1e-8)
    best, best_s = math.inf, torch.ones_like(mean)
    for j in range(grid_points):
        a = j / grid_points
        s = mean.pow(a).clamp(min=1e-4)
        s = s / (s.max() * s.min()).sqrt()
        loss = _awq_loss(x, w, s, fmt, group, symmetric)
        if loss < best:
            best, best_s = loss, s
    return best_s


@torch.no_grad()
def awq_clip(weight: torch.Tensor, x: torch.Tensor, fmt: str, group: int, symmetric: bool,
             grid_points: int, max_shrink: float = 0.5) -> torch.Tensor:
    """Per (row, group) clipping ratio minimising the group's output error on the sample ``x``."""
    group = FP4_GROUP.get(fmt, group)
    w = _groups(weight.float(), group)  # [N, G, g]
    xg = x.float().reshape(x.shape[0], -1, group)  # [T, G, g]
    ref = torch.einsum("ngk,tgk->ngt", w, xg)
    best = torch.full(w.shape[:2], math.inf, device=w.device)
    ratio = torch.ones(w.shape[:2], device=w.device)
    steps = max(1, int(grid_points * max_shrink))
    for j in range(steps):
        r = 1.0 - j / grid_points
        grid = fit_grid(w, fmt, symmetric, r)
        _, dq = quantize_codes(w, grid, fmt)
        err = (torch.einsum("ngk,tgk->ngt", dq, xg) - ref).pow(2).mean(-1)
        better = err < best
        best = torch.where(better, err, best)
        ratio = torch.where(better, torch.full_like(ratio, r), ratio)
    return ratio


QUANTIZERS: dict[str, Callable] = {"rtn": rtn, "gptq": gptq}


# ---- HQQ ------------------------------------------------------------------------------------------------------
def _shrink_lp(x: torch.Tensor, beta: float, p: float) -> torch.Tensor:
    """The generalised soft-thresholding of the ``l_p`` proximal step (HQQ, Badri & Shaji 2023)."""
    return torch.sign(x) * torch.relu(x.abs() - (1.0 / beta) * x.abs().clamp_min(1e-8).pow(p - 1))


@torch.no_grad()
def hqq(weight: torch.Tensor, fmt: str, group: int | None, symmetric: bool, iters: int = 20, p: float = 0.7,
        beta: float = 10.0, kappa: float = 1.01) -> QWeight:
    """Half-quadratic quantization: from the min-max grid, alternate ``W_e = shrink_lp(W - W_r)`` (the sparse error
    the ``l_p`` model tolerates) with the grid that fits ``W - W_e``: the zero point (rounded to the stored integer
    grid) and, by least squares, the scale. Calibration-free."""
    g = group or weight.shape[1]
    w = _groups(weight.float(), g)
    grid = fit_grid(w, fmt, symmetric)
    if fmt not in _INT_TOP:
        codes, _ = quantize_codes(w, grid, fmt)
        return _qweight(codes, grid, fmt, g, weight.dtype)
    top = _INT_TOP[fmt]
    best_err = (quantize_codes(w, grid, fmt)[1] - w).pow(2).sum(-1)
    best = Grid(grid.scale.clone(), grid.zero.clone())
    s, z = grid.scale.clone(), grid.zero.clone()
    for _ in range(iters):
        q = torch.clamp(torch.round(w / s[..., None]) + z[..., None], 0, top)
        w_r = (q - z[..., None]) * s[..., None]
        w_e = _shrink_lp(w - w_r, beta, p)
        target = w - w_e
        if not symmetric:
            z = torch.round((q - target / s[..., None]).mean(-1)).clamp(0, top)
        c = q - z[..., None]
        s = ((c * target).sum(-1) / c.pow(2).sum(-1).clamp_min(1e-12)).clamp_min(1e-8).to(torch.bfloat16).float()
        beta *= kappa
        cand = Grid(s, z)
        err = (quantize_codes(w, cand, fmt)[1] - w).pow(2).sum(-1)
        better = err < best_err
        best.scale = torch.where(better, s, best.scale)
        best.zero = torch.where(better, z, best.zero)
        best_err = torch.minimum(err, best_err)
    codes, _ = quantize_codes(w, best, fmt)
    return _qweight(codes, best, fmt, g, weight.dtype)


# ---- SmoothQuant ----------------------------------------------------------------------------------------------
@torch.no_grad()
def smooth_scales(weights: Sequence[torch.Tensor], stats: _Stats, alpha: float) -> torch.Tensor:
    """SmoothQuant's per-input-channel scale ``s_j = max|X_j|^alpha / max|W_j|^(1 - alpha)`` (Xiao et al., 2023):
    the activations are divided by ``s`` (folded into their producer) and the weights multiplied by it."""
    x_max = stats.sample.abs().amax(0).clamp_min(1e-5)
    w_max = torch.cat([w.float() for w in weights], 0).abs().amax(0).clamp_min(1e-5)
    return (x_max.pow(alpha) / w_max.pow(1.0 - alpha)).clamp_min(1e-5)
