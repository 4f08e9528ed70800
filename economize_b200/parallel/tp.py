"""Tensor parallelism of the engine's decoder (Megatron-style sharding of the fused weights).

Rank ``r`` of ``P`` keeps query heads ``[r*H/P, (r+1)*H/P)`` and KV heads ``[r*Hkv/P, (r+1)*Hkv/P)`` of the fused
QKV projection, the matching input columns of ``wo`` (row-parallel), features ``[r*F/P, (r+1)*F/P)`` of gate and up
and the matching columns of ``w_down``, and vocabulary rows ``[r*V/P, (r+1)*V/P)`` of the LM head. Norms, the
embedding and drafters are replicated. Every rank therefore holds identical residual streams after each
all-reduce, computes identical draft trees and acceptance decisions, and no control data is broadcast.

The two row-parallel projections of a block end in a reduction of ``[tokens, hidden]`` over the ranks. With NCCL
(the baseline) it is an all-reduce of the full rows. With ``fused=True`` a pass runs sequence-parallel through
:mod:`economize_b200.parallel.sp`: the row-parallel GEMM stores every output row into its owner rank's slot over
NVLink (GEMM -> reduce-scatter), the owner sums the ranks' partials in rank order, adds the residual, applies the
next RMSNorm and pushes the normed rows to every rank, and the next column-parallel GEMM waits for them
(all-gather -> GEMM); every rank gets bit-identical rows.
Economize relies on ``transformers``' ``tp_plan="auto"`` with DTensor (``src/economize/distributed/tp.py:117-138``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..errors import ConfigError

__all__ = ["TPGroup", "shard_model", "tp_argmax"]


@dataclass
class TPGroup:
    """A tensor-parallel group: rank, size, process group, and the fused-collective runtime when enabled."""

    rank: int
    size: int
    group: object = None
    fused: bool = False
    comm: object = None
    #: the sequence-parallel fused collectives (parallel/sp.py); passes they cannot carry take NCCL
    sp: object = None

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return x
        dist.all_reduce(x, group=self.group)
        return x

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        """``[size, *x.shape]`` of every rank's ``x``."""
        x = x.contiguous()
        if x.is_cuda:
            out = torch.empty((self.size, *x.shape), dtype=x.dtype, device=x.device)
            dist.all_gather_into_tensor(out, x, group=self.group)
            return out
        parts = [torch.empty_like(x) for _ in range(self.size)]
        dist.all_gather(parts, x, group=self.group)
        return torch.stack(parts)


def _split(n: int, parts: int, what: str) -> int:
    if n % parts:
        raise ConfigError(f"{what} ({n}) does not split over {parts} tensor-parallel ranks")
    return n // parts


@torch.no_grad()
def shard_model(model, tp: TPGroup):
    """Shard an engine :class:`~economize_b200.models.CausalLM` in place for rank ``tp.rank`` of ``tp.size``."""
    if tp.size == 1:
        model.tp = tp
        return model
    c = model.config
    if c.is_moe:
        raise ConfigError("tensor parallelism of MoE blocks is expert parallelism (economize_b200.parallel.ep)")
    r, p = tp.rank, tp.size
    hq, hkv, f, v = _split(c.num_heads, p, "query heads"), _split(c.num_kv_heads, p, "KV heads"), \
        _split(c.intermediate_size, p, "FFN width"), _split(c.vocab_size, p, "vocabulary")
    d = c.head_dim
    for layer in model.layers:
        q, k, vv = layer.wqkv.data.split([c.q_size, c.kv_size, c.kv_size], 0)
        layer.wqkv.data = torch.cat([q[r * hq * d:(r + 1) * hq * d], k[r * hkv * d:(r + 1) * hkv * d],
                                     vv[r * hkv * d:(r + 1) * hkv * d]], 0).contiguous()
        if layer.bqkv is not None:
            bq, bk, bv = layer.bqkv.data.split([c.q_size, c.kv_size, c.kv_size], 0)
            layer.bqkv.data = torch.cat([bq[r * hq * d:(r + 1) * hq * d], bk[r * hkv * d:(r + 1) * hkv * d],
                                         bv[r * hkv * d:(r + 1) * hkv * d]], 0).contiguous()
        layer.wo.data = layer.wo.data[:, r * hq * d:(r + 1) * hq * d].contiguous()
        if layer.sinks is not None:  # one sink logit per query head: this rank's heads
            layer.sinks.data = layer.sinks.data[r * hq:(r + 1) * hq].contiguous()
        gate, up = layer.w_gate_up.data.chunk(2, 0)
        layer.w_gate_up.data = torch.cat([gate[r * f:(r + 1) * f], up[r * f:(r + 1) * f]], 0).contiguous()
        if layer.down_hadamard and f % layer.down_hadamard:
            raise ConfigError(f"the online Hadamard block {layer.down_hadamard} of the down projection does not "
                              f"divide the per-rank width {f}; rotate with a smaller block")
        layer.w_down.data = layer.w_down.data[:, r * f:(r + 1) * f].contiguous()
    if model.lm_head is None:
        model.lm_head = torch.nn.Parameter(model.embed.data[r * v:(r + 1) * v].clone())
        c.tie_word_embeddings = False
    else:
        model.lm_head.data = model.lm_head.data[r * v:(r + 1) * v].contiguous()
    model.tp = tp
    model.local = dict(num_heads=hq, num_kv_heads=hkv, intermediate_size=f, vocab_offset=r * v, vocab_size=v)
    return model


def tp_argmax(local_logits: torch.Tensor, tp: TPGroup, vocab_offset: int) -> torch.Tensor:
    """Global argmax over vocabulary shards: every rank exchanges its rows' (max, index) pairs; ties go to the
    smallest global index, as a single-device argmax does."""
    from .. import ops

    idx = ops.argmax(local_logits)
    val = local_logits.gather(-1, idx[..., None])[..., 0].float()
    pairs = torch.stack([val, (idx + vocab_offset).float()], -1)  # exact for vocabularies below 2**24
    every = tp.all_gather(pairs)  # [P, ..., 2]
    best = every[..., 0].amax(0, keepdim=True)
    cand = torch.where(every[..., 0] == best, every[..., 1], torch.full_like(every[..., 1], float("inf")))
    return cand.amin(0).long()
