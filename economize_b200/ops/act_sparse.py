"""Activation sparsity shared by TEAL, CATS and Deja Vu: phase policies, magnitude thresholds, TEAL's greedy
allocation, and the weight and MLP objects that route decoding steps to the sparse kernels of
``csrc/act_sparse.cu`` (economize ``techniques/sparsity/sparsify.py``, ``techniques/mlp_sparsity/mlp.py``).

* :class:`TransposedWeight` stores a ``[out, in]`` weight as row-major ``W^T`` (the storage is replaced, not
  duplicated). Column-sparse products stream only the rows of ``W^T`` whose input is kept
  (``colsparse_linear``); every other call runs the dense product on the transposed storage.
* :class:`TealWeight` adds TEAL's threshold and phase policy: decoding calls of at most :data:`MAX_ROWS` rows that
  the policy sparsifies in full run the kernel; the rest run ``linear(sparsify(x), W)``.
* :func:`cats_mlp` and :func:`kept_mlp` are the CATS and Deja Vu MLP forwards: ``glu_rows`` reads only the up (and
  gate) rows of kept channels, the down projection is column-sparse over the exact zeros of its input.
"""

from __future__ import annotations

from collections.abc import Callable, Mapping
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from ..errors import ConfigError
from ..runtime.phase import current_phase

__all__ = ["MAX_ROWS", "POLICY_PHASES", "PREFILL_MODES", "GreedyStep", "PhasePolicy", "TealWeight", "TransposedWeight",
           "apply_mode", "block_sparsity", "cats_mlp", "greedy_allocation", "greedy_error", "kept_channels",
           "kept_mlp", "magnitude_quantile", "sparsify", "topk_mask", "uniform_allocation"]

#: Most rows (tokens x sequences) a call may have to run the sparse kernels: from about four independent rows on,
#: their union keeps nearly every column and the dense GEMM is faster.
MAX_ROWS = 4

#: How a forward call's tokens are treated: ``"dense"`` unchanged, ``"second_half"`` the last ``max(1, S // 2)``
#: positions of every sequence are sparsified (TEAL's perplexity protocol), ``"all"`` every position.
PREFILL_MODES = ("dense", "second_half", "all")


#: The kinds of forward call a :class:`PhasePolicy` distinguishes (the engine's phases, plus calls outside it).
POLICY_PHASES = ("prefill", "refresh", "decode", "draft", "outside")


@dataclass(frozen=True)
class PhasePolicy:
    """The mode (:data:`PREFILL_MODES`) of each kind of forward call, by decoding phase
    (:mod:`economize_b200.runtime.phase`). The default sparsifies decoding and drafting steps and keeps the exact
    passes dense; calls outside the engine with one token per sequence follow ``decode``, longer ones ``outside``
    (economize ``techniques/sparsity/sparsify.py:47-110``)."""

    prefill: str = "dense"
    refresh: str = "dense"
    decode: str = "all"
    draft: str = "all"
    outside: str = "dense"

    def __post_init__(self) -> None:
        for phase in POLICY_PHASES:
            mode = getattr(self, phase)
            if mode not in PREFILL_MODES:
                raise ConfigError(f"PhasePolicy.{phase}={mode!r} is not a mode; use one of {', '.join(PREFILL_MODES)}")

    @classmethod
    def from_prefill(cls, mode: str) -> PhasePolicy:
        """The policy of ``prefill=mode``: the exact passes and multi-token calls outside decoding follow ``mode``."""
        return cls(**{phase: mode for phase in ("prefill", "refresh", "outside")})

    @classmethod
    def coerce(cls, value) -> PhasePolicy:
        """A policy from itself, a mode name (:meth:`from_prefill`) or a mapping of phase to mode."""
        if isinstance(value, cls):
            return value
        if isinstance(value, str):
            if value in PREFILL_MODES:
                return cls.from_prefill(value)
            raise ConfigError(f"{value!r} names no mode; a prefill mode is one of {', '.join(PREFILL_MODES)}")
        if isinstance(value, Mapping):
            extra = [key for key in value if key not in POLICY_PHASES]
            if extra:
                raise ConfigError(f"a phase policy maps the phases {', '.join(POLICY_PHASES)} to modes; "
                                  f"{sorted(extra)} are not phases")
            return cls(**dict(value))
        raise ConfigError(f"cannot read a phase policy from {type(value).__name__} {value!r}")

    def to_dict(self) -> dict[str, str]:
        return {phase: getattr(self, phase) for phase in POLICY_PHASES}

    def mode(self, phase: str | None, tokens: int | None) -> str:
        """The mode of a call in ``phase`` over ``tokens`` positions per sequence."""
        if phase is not None:
            return str(getattr(self, phase))
        return self.decode if tokens == 1 else self.outside


def tokens_per_sequence(x: torch.Tensor) -> int | None:
    """Positions per sequence of a map input ``[B, S, D]`` (``None`` for a flat input)."""
    return x.shape[-2] if x.dim() >= 3 else None


def sparsify(x: torch.Tensor, threshold: torch.Tensor | float) -> torch.Tensor:
    """TEAL's ``x * 1[|x| > t]`` (a 0-dim fp32 threshold is compared in ``x``'s dtype, as PyTorch promotes)."""
    return x * (x.abs() > threshold)


def second_half_mask(keep: torch.Tensor) -> torch.Tensor:
    """``keep`` with every entry of the first ``S - max(1, S // 2)`` positions of every sequence set."""
    if keep.dim() < 2:
        return keep
    half = max(1, keep.shape[-2] // 2)
    keep = keep.clone()
    keep[..., : keep.shape[-2] - half, :] = True
    return keep


def apply_mode(x: torch.Tensor, threshold: torch.Tensor | float, mode: str) -> torch.Tensor:
    """``x`` sparsified as ``mode`` says."""
    if mode == "dense":
        return x
    if mode == "all" or x.dim() < 2:
        return sparsify(x, threshold)
    return x * second_half_mask(x.abs() > threshold)


def magnitude_quantile(sorted_magnitudes: torch.Tensor, q: float) -> float:
    """The ``q``-quantile of ascending magnitudes (lower interpolation): the threshold that drops a fraction ``q``
    (``q = 0`` gives 0: only exact zeros are dropped)."""
    n = sorted_magnitudes.numel()
    if q <= 0 or n == 0:
        return 0.0
    k = min(n, max(1, round(q * n)))
    return float(sorted_magnitudes[k - 1])


def block_sparsity(sparsities: Mapping[str, float], sizes: Mapping[str, int]) -> float:
    """Parameter-weighted mean sparsity of a layer's maps: the fraction of its weight reads a sparse kernel skips."""
    names = list(sizes)
    weights = [sizes[n] for n in names]
    skipped = sum(w * sparsities[n] for n, w in zip(names, weights))
    return skipped / max(sum(weights), 1)


def uniform_allocation(sizes: Mapping[str, int], target: float) -> dict[str, float]:
    """Every map of the layer at the same sparsity ``target``."""
    return {name: target for name in sizes}


@dataclass(frozen=True)
class GreedyStep:
    """One move of :func:`greedy_allocation`: the map that was raised, the layer's sparsity after the move and
    the layer error the move measured."""

    name: str
    block_sparsity: float
    error: float


def greedy_allocation(error: Callable[[Mapping[str, float]], float], sizes: Mapping[str, int], target: float, *,
                      step: float = 0.05, unit: int | None = None) -> tuple[dict[str, float], list[GreedyStep]]:
    """TEAL's block-wise greedy allocation (Liu et al., 2025, Algorithm 1).

    Every map's sparsity moves in increments sized so that one increment of any map adds ``step * unit / total``
    to the layer's weighted sparsity (``unit``: the largest map's size by default). Each round evaluates ``error``
    on every map raised by one increment and keeps the cheapest move; rounds continue until the layer reaches
    ``target`` or no map can move. Returns the sparsities and the moves in order.
    """
    scale = unit if unit else max(sizes.values())
    increment = {name: step * scale / size for name, size in sizes.items()}
    count = {name: 0 for name in sizes}

    def level(name: str, extra: int = 0) -> float:
        return min(1.0, (count[name] + extra) * increment[name])

    def levels(raise_one: str | None = None) -> dict[str, float]:
        return {name: level(name, 1 if name == raise_one else 0) for name in sizes}

    history: list[GreedyStep] = []
    current = levels()
    while block_sparsity(current, sizes) + 1e-9 < target:
        movable = [name for name in sizes if level(name) < 1.0]
        if not movable:
            break
        trials = [(error(levels(name)), position, name) for position, name in enumerate(movable)]
        cost, _, chosen = min(trials)
        count[chosen] += 1
        current = levels()
        history.append(GreedyStep(chosen, block_sparsity(current, sizes), cost))
    return current, history


def greedy_error(reference: torch.Tensor, output: torch.Tensor, fraction: float = 0.25) -> float:
    """L2 norm over the last ``fraction`` of the positions of ``reference - output`` ``[B, S, D]``, averaged over
    batch and hidden dimension (TEAL's layer error)."""
    start = int(output.shape[1] * (1 - fraction))
    return float(torch.linalg.vector_norm((reference[:, start:] - output[:, start:]).float(), dim=1).mean())


def kept_channels(ffn: int, sparsity: float) -> int:
    """FFN channels computed per token at ``sparsity`` (at least one)."""
    return max(1, round((1.0 - sparsity) * ffn))


def topk_mask(scores: torch.Tensor, k: int) -> torch.Tensor:
    index = scores.topk(k, dim=-1).indices
    return torch.zeros(scores.shape, dtype=torch.bool, device=scores.device).scatter_(-1, index, True)


def _kernels_usable(x: torch.Tensor, rows: int) -> bool:
    return x.is_cuda and x.dtype == torch.bfloat16 and 0 < rows <= MAX_ROWS


def _dense_linear(x: torch.Tensor, weight) -> torch.Tensor:
    from . import linear

    return linear(x, weight)


class TransposedWeight(nn.Module):
    """A ``[out, in]`` weight stored as row-major ``W^T [in, out]`` for column-sparse products.

    :meth:`linear` is the dense product on the transposed storage (cuBLAS on CUDA, which reads either layout);
    :meth:`sparse_linear` streams only the rows of ``W^T`` whose input column is kept (``colsparse_linear``)."""

    def __init__(self, weight: torch.Tensor) -> None:
        super().__init__()
        self.register_buffer("weight_t", weight.detach().t().contiguous())

    @property
    def shape(self) -> torch.Size:
        return torch.Size((self.weight_t.shape[1], self.weight_t.shape[0]))

    @property
    def dtype(self) -> torch.dtype:
        return self.weight_t.dtype

    @property
    def device(self) -> torch.device:
        return self.weight_t.device

    def dequantize(self, dtype: torch.dtype | None = None) -> torch.Tensor:
        w = self.weight_t.t()
        return w if dtype is None else w.to(dtype)

    def restore(self) -> torch.Tensor:
        """The weight in the usual ``[out, in]`` row-major layout."""
        return self.weight_t.t().contiguous()

    def linear(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x, self.weight_t.t().to(x.dtype))

    def sparse_linear(self, x: torch.Tensor, threshold: torch.Tensor | None = None) -> torch.Tensor:
        """``sparsify(x, threshold) @ W^T`` (no threshold: the exact zeros of ``x`` are skipped)."""
        rows = x.numel() // x.shape[-1]
        if _kernels_usable(x, rows) and self.weight_t.dtype == torch.bfloat16:
            from ._ext import require

            return require().colsparse_linear(x, self.weight_t, threshold)
        return self.linear(x if threshold is None else sparsify(x, threshold))


class TealWeight(nn.Module):
    """A linear map under TEAL: ``linear(x)`` sparsifies the input as the phase policy says.

    With ``kernel`` the weight is stored transposed and the calls that the policy sparsifies in full with at most
    :data:`MAX_ROWS` rows run ``colsparse_linear`` (only the weight rows of kept inputs are read); every other call
    computes ``linear(sparsify(x), W)``. Without ``kernel`` the weight keeps its layout (or stays the object it
    was, e.g. a quantized weight) and every call is the masked dense product (a simulation of the saving).
    """

    def __init__(self, weight, threshold: float, policy: PhasePolicy, kernel: bool) -> None:
        super().__init__()
        self.kernel = bool(kernel)
        self.policy = policy
        device = weight.device
        if self.kernel:
            self.register_buffer("weight_t", weight.detach().t().contiguous())
            self.inner = None
        elif isinstance(weight, torch.Tensor):
            self.register_buffer("weight", weight.detach())
            self.inner = None
        else:
            self.inner = weight  # a weight object with its own ``linear`` (quantized, 2:4, ...)
        self.register_buffer("threshold", torch.tensor(float(threshold), dtype=torch.float32, device=device))

    @property
    def shape(self) -> torch.Size:
        if self.kernel:
            return torch.Size((self.weight_t.shape[1], self.weight_t.shape[0]))
        return self.inner.shape if self.inner is not None else self.weight.shape

    @property
    def dtype(self) -> torch.dtype:
        if self.kernel:
            return self.weight_t.dtype
        return self.inner.dtype if self.inner is not None else self.weight.dtype

    @property
    def device(self) -> torch.device:
        return self.threshold.device

    def restore(self):
        """The wrapped weight in its original form (``[out, in]`` tensor, or the wrapped object)."""
        if self.kernel:
            return self.weight_t.t().contiguous()
        return self.inner if self.inner is not None else self.weight

    def dequantize(self, dtype: torch.dtype | None = None) -> torch.Tensor:
        w = self.restore()
        w = w if isinstance(w, torch.Tensor) else w.dequantize()
        return w if dtype is None else w.to(dtype)

    def _dense(self, x: torch.Tensor) -> torch.Tensor:
        if self.kernel:
            return F.linear(x, self.weight_t.t())
        return _dense_linear(x, self.inner if self.inner is not None else self.weight)

    def linear(self, x: torch.Tensor) -> torch.Tensor:
        mode = self.policy.mode(current_phase(), tokens_per_sequence(x))
        if mode == "dense":
            return self._dense(x)
        if mode == "all" and self.kernel and _kernels_usable(x, x.numel() // x.shape[-1]):
            from ._ext import require

            return require().colsparse_linear(x, self.weight_t, self.threshold)
        return self._dense(apply_mode(x, self.threshold, mode))


def _down(h: torch.Tensor, down, sparse: bool) -> torch.Tensor:
    if isinstance(down, TransposedWeight):
        return down.sparse_linear(h) if sparse else down.linear(h)
    return _dense_linear(h, down)


def cats_mlp(w_gate_up, down, x: torch.Tensor, threshold: torch.Tensor, mode: str, kernel: bool) -> torch.Tensor:
    """CATS's gated MLP ``down((g * 1[|g| > t]) * up(x))`` with ``g = silu(gate(x))`` (Lee et al., 2024, Eq. 2):
    with ``kernel`` a decoding call reads only the up rows and down columns of kept channels."""
    rows = x.numel() // x.shape[-1]
    if mode == "all" and kernel and _kernels_usable(x, rows) and isinstance(w_gate_up, torch.Tensor):
        from ._ext import require

        f = w_gate_up.shape[0] // 2
        gate = _dense_linear(x, w_gate_up[:f])
        h = require().glu_rows(x, w_gate_up, gate, None, threshold)
        return _down(h, down, True)
    gate, up = _dense_linear(x, w_gate_up).chunk(2, -1)
    g = F.silu(gate)
    keep = g.abs() > threshold
    if mode == "second_half":
        keep = second_half_mask(keep)
    return _down(g.masked_fill(~keep, 0) * up, down, False)


def kept_mlp(w_gate_up, down, x: torch.Tensor, keep: torch.Tensor, kernel: bool) -> torch.Tensor:
    """The gated MLP computed on the channels in ``keep [..., F]`` only (Deja Vu): with ``kernel`` a decoding call
    reads only the gate and up rows and down columns of kept channels."""
    rows = x.numel() // x.shape[-1]
    if kernel and _kernels_usable(x, rows) and isinstance(w_gate_up, torch.Tensor):
        from ._ext import require

        h = require().glu_rows(x, w_gate_up, None, keep, None)
        return _down(h, down, True)
    gate, up = _dense_linear(x, w_gate_up).chunk(2, -1)
    g = F.silu(gate).masked_fill(~keep, 0)
    return _down(g * up.masked_fill(~keep, 0), down, False)
