"""SliceGPT (``slicegpt``; Ashkboos et al., 2024; economize ``techniques/slicegpt``): rotate the residual stream
into its principal components and delete the least significant ones, shrinking the hidden width.

The RMSNorm weights are folded into the projections that read them (after which the network is invariant to an
orthogonal ``Q`` on the residual stream, as in ``rotate``); ``Q`` holds the eigenvectors of the normalised residual
streams' covariance summed over every block input on calibration text, in decreasing order, and only its first
``d = (1 - sparsity) H`` columns are kept (``d`` rounded up to ``round_to``): ``embed' = embed Q_d``, readers
``W' = W Q_d`` (QKV, gate/up, LM head), writers ``W' = Q_d^T W`` (o, down). The norms then run over ``d`` channels;
their weights become ``sqrt(H / d)``, which keeps the normalised scale of streams whose energy lies in the kept
components. The engine's kernels run the narrower model unchanged.

Rotation ``"global"`` (one basis for every block) is built; economize's default ``"per_block"`` needs a transform on
the residual shortcut between blocks, which the engine's fused residual-add + norm does not have (ConfigError).
The technique refuses tensor parallelism (rotate before sharding).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import ClassVar

import torch
from torch import nn

from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...errors import ConfigError
from ...runtime.cache import StepBatch
from ...validation import check_choice, check_positive, check_unit_interval

__all__ = ["SliceGPTConfig", "SliceGPTTechnique", "pca_basis"]


@dataclass(frozen=True)
class SliceGPTConfig(TechniqueConfig):
    technique: ClassVar[str] = "slicegpt"
    sparsity: float = 0.25
    rotation: str = "global"
    slice_head: bool | None = None
    round_to: int = 128
    offload: bool = False

    def __post_init__(self) -> None:
        check_unit_interval("sparsity", self.sparsity, closed_low=True)
        if self.rotation == "per_block":
            raise ConfigError("slicegpt rotation='per_block' needs a transform on the residual shortcut between "
                              "blocks; this engine fuses the residual add into the norm: use rotation='global'")
        check_choice("rotation", self.rotation, ("global",))
        check_positive("round_to", self.round_to)

    def width(self, hidden: int) -> int:
        d = math.ceil((1.0 - self.sparsity) * hidden / self.round_to) * self.round_to
        return max(self.round_to, min(hidden, d))


@torch.no_grad()
def pca_basis(model, batches) -> torch.Tensor:
    """Eigenvectors (columns, decreasing eigenvalue) of the summed covariance of the RMS-normalised residual stream
    at every block input and after the last block."""
    n = model.config.num_layers
    h = model.config.hidden_size
    cov = torch.zeros(h, h, dtype=torch.float64, device=model.device)
    for tokens in batches:
        tokens = tokens.to(model.device)
        if tokens.dim() == 1:
            tokens = tokens[None]
        b, s = tokens.shape
        cache = model.new_cache(b, ((s + 127) // 128) * 128)
        lengths = torch.full((b,), s, dtype=torch.int32, device=model.device)
        _, aux = model.forward_step(tokens, StepBatch.prefill(lengths, s), cache, capture=tuple(range(n + 1)))
        for i in range(n + 1):
            x = aux[i].reshape(-1, h).double()
            x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)
            cov += x.t() @ x
    evals, evecs = torch.linalg.eigh(cov)
    order = torch.argsort(evals, descending=True)
    return evecs[:, order].float()


@register_technique
class SliceGPTTechnique(Technique):
    """State: ``basis [H, d]`` (the kept rotation columns), so a saved model re-slices without calibration."""

    config_class = SliceGPTConfig
    capabilities = Capability.WEIGHTS
    family = Family.PRUNING
    lossless = False

    def __init__(self, config: SliceGPTConfig, model) -> None:
        super().__init__(config, model)
        if model.config.is_moe:
            raise ConfigError("slicegpt supports dense models")
        self.hidden = model.config.hidden_size
        self.register_buffer("basis", torch.zeros(0, device=model.device))
        self._calibration = None
        self.applied = False

    def calibrate(self, calibration) -> None:
        self._calibration = calibration

    @torch.no_grad()
    def attach(self) -> None:
        if self.applied:
            return
        m = self.model
        if m.tp is not None and m.tp.size > 1:
            raise ConfigError("slicegpt refuses tensor parallelism: slice before sharding")
        if self.basis.numel() == 0:
            cal = self._calibration
            if cal is None:
                raise ConfigError("slicegpt needs calibration tokens (apply(..., calibration=ids)) or a saved state")
            batches = [cal] if isinstance(cal, torch.Tensor) else list(cal)
            d = self.config.width(self.hidden)
            self.basis = pca_basis(m, batches)[:, :d].contiguous()
        q = self.basis.to(m.device).float()
        d = q.shape[1]
        dt = m.dtype
        if m.lm_head is None:
            m.lm_head = nn.Parameter(m.embed.detach().clone())
            m.config.tie_word_embeddings = False

        def put(owner, name: str, value: torch.Tensor) -> None:
            setattr(owner, name, nn.Parameter(value.to(dt).contiguous(), requires_grad=False))

        scale = math.sqrt(self.hidden / d)
        for layer in m.layers:
            put(layer, "wqkv", (layer.wqkv.float() * layer.attn_norm.float()[None]) @ q)
            put(layer, "w_gate_up", (layer.w_gate_up.float() * layer.mlp_norm.float()[None]) @ q)
            put(layer, "wo", q.t() @ layer.wo.float())
            put(layer, "w_down", q.t() @ layer.w_down.float())
            put(layer, "attn_norm", torch.full((d,), scale, device=m.device))
            put(layer, "mlp_norm", torch.full((d,), scale, device=m.device))
        put(m, "lm_head", (m.lm_head.float() * m.norm.float()[None]) @ q)
        put(m, "norm", torch.full((d,), scale, device=m.device))
        put(m, "embed", m.embed.float() @ q)
        import dataclasses

        m.config = dataclasses.replace(m.config, hidden_size=d)
        m._rope = None
        self.applied = True

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        unknown = sorted(set(state) - {"basis"})
        if unknown:
            raise ConfigError(f"slicegpt: unexpected tensors {unknown[:5]}")
        if "basis" in state:
            self.basis = state["basis"].to(self.model.device).float().contiguous()

    def parameter_ratio(self) -> float:
        """Projection parameters kept (``d / H`` of every projection's hidden side)."""
        return self.basis.shape[1] / self.hidden if self.basis.numel() else 1.0
