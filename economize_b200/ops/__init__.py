"""Operators of the decode engine.

Every operator takes the hand-written sm_100a kernel of ``economize_b200._C`` for CUDA tensors and the PyTorch
implementation of :mod:`.reference` for CPU tensors. There is no third path: a CUDA tensor with the extension
missing raises :class:`~economize_b200.errors.KernelUnavailableError`.
"""

from __future__ import annotations

import torch

from . import reference
from ._ext import available, load_error, require
from .fp8 import FP8BlockWeight
from .quant import QWeight
from .sparse import Sparse24Weight

__all__ = [
    "argmax",
    "attention",
    "attention_scores",
    "attention_usage",
    "available",
    "greedy_accept",
    "kivi_quantize",
    "kv_compact",
    "linear",
    "linear_parts",
    "Partials",
    "load_error",
    "require",
    "rmsnorm",
    "ngram",
    "QWeight",
    "rejection",
    "rope_store",
    "sample",
    "topk_logp",
    "tree_layout",
    "silu_mul",
    "hadamard",
    "vs_keep",
    "gelu_tanh_mul",
    "glu",
]


class Partials:
    """Split-K partial products ``data [splits, ..., N]`` (fp32) of a projection whose consumer sums them (in split
    order, rounded to bf16: the value the GEMM would have stored) instead of the GEMM reducing them itself."""

    __slots__ = ("data",)

    def __init__(self, data: torch.Tensor) -> None:
        self.data = data

    @property
    def shape(self) -> torch.Size:
        return self.data.shape[1:]

    @property
    def is_cuda(self) -> bool:
        return True

    @property
    def dtype(self) -> torch.dtype:
        return torch.bfloat16  # the dtype of the tensor the partials stand for

    @property
    def device(self) -> torch.device:
        return self.data.device

    def __getitem__(self, index) -> Partials:
        """Index the represented tensor (the split dimension is kept)."""
        index = index if isinstance(index, tuple) else (index,)
        return Partials(self.data[(slice(None),) + index].contiguous())

    def numel(self) -> int:
        return self.data[0].numel()

    def sum(self) -> torch.Tensor:
        """The bf16 tensor the partials stand for."""
        acc = self.data[0].clone()
        for i in range(1, self.data.shape[0]):
            acc += self.data[i]
        return acc.to(torch.bfloat16)


def _raw(x):
    return x.data if isinstance(x, Partials) else x


def linear_parts(x: torch.Tensor, weight) -> torch.Tensor | Partials:
    """``x @ weight.T`` for a consumer that fuses the split-K reduction (:func:`rmsnorm`, :func:`silu_mul`,
    :func:`rope_store`): :class:`Partials` on CUDA when the GEMM splits K, else the plain result."""
    if not x.is_cuda or not isinstance(weight, torch.Tensor) or x.dtype != torch.bfloat16:
        return linear(x, weight)
    shape = x.shape
    y = require().linear_parts(x.reshape(-1, shape[-1]), weight)
    if y.dtype == torch.bfloat16:
        return y.reshape(*shape[:-1], weight.shape[0])
    return Partials(y.reshape(y.shape[0], *shape[:-1], weight.shape[0]))


def rmsnorm(x: torch.Tensor | Partials, weight: torch.Tensor, eps: float,
            residual: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused residual add + RMSNorm: ``(norm(x + residual) * weight, x + residual)`` over the last dim."""
    if x.is_cuda:
        return require().rmsnorm(_raw(x), weight, float(eps), residual)
    return reference.rmsnorm(x, weight, eps, residual)


def rope_store(qkv: torch.Tensor, positions: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, num_heads: int,
               num_kv_heads: int, head_dim: int, k_cache: torch.Tensor, v_cache: torch.Tensor,
               kv_len: torch.Tensor, n_new: torch.Tensor, q_norm: torch.Tensor | None = None,
               k_norm: torch.Tensor | None = None, eps: float = 1e-6, q_offset: int = 0,
               k_scale: torch.Tensor | None = None, v_scale: torch.Tensor | None = None,
               pages: torch.Tensor | None = None) -> torch.Tensor:
    """Fused (per-head RMSNorm +) rotary embedding of queries and keys and the KV-cache write (see
    :func:`.reference.rope_store`); fp8 caches are written as e4m3 codes of ``value / scale``; ``pages``: paged
    caches (as for :func:`attention`)."""
    if qkv.is_cuda:
        return require().rope_store(_raw(qkv), positions, cos, sin, num_heads, num_kv_heads, head_dim, k_cache, v_cache,
                                    kv_len, n_new, q_norm, k_norm, float(eps), int(q_offset), k_scale, v_scale, pages)
    return reference.rope_store(qkv, positions, cos, sin, num_heads, num_kv_heads, head_dim, k_cache, v_cache,
                                kv_len, n_new, q_norm, k_norm, eps, q_offset, k_scale, v_scale, pages)


def attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, kv_len: torch.Tensor,
              n_new: torch.Tensor, mask: torch.Tensor | None = None, scale: float | None = None,
              q_offset: int = 0, k_scale: torch.Tensor | None = None,
              v_scale: torch.Tensor | None = None, keep: torch.Tensor | None = None,
              lse_out: torch.Tensor | None = None, kivi: torch.Tensor | None = None,
              kivi_chunks: torch.Tensor | None = None, kivi_bits: int = 0, tail: int = 0,
              softcap: float | None = None, sinks: torch.Tensor | None = None, window: int = 0,
              pages: torch.Tensor | None = None) -> torch.Tensor:
    """Causal / tree-masked attention over the slot cache (see :func:`.reference.attention`); fp8 caches take
    per-KV-head scales, ``keep`` (int32 bit words ``[B, H_kv, S / 32]``) hides evicted committed slots and
    ``lse_out [B, T, H]`` receives every row's log2-domain log-sum-exp. ``softcap`` (tanh soft-capping of the
    scores), ``sinks`` (fp32 ``[H]`` sink logits) and ``window`` (sliding window in positions; the kernel then reads
    only the window's chunks) serve Gemma-2, gpt-oss and the sliding-window layers of Mistral, Gemma-2/3 and OLMo-3.
    ``pages [B, C]`` (int32): the caches are views ``[P, H_kv, 128, D]`` of a page pool and logical chunk ``c`` of row
    ``b`` is page ``pages[b, c]`` (:class:`~economize_b200.runtime.cache.PagedKVCache`).

    ``tail > 0`` (passes of at most 64 queries) reduces the keys at the last ``tail`` positions before each query,
    and its own new keys, one at a time in position order: a verification pass then computes every query bit for
    bit as a one-token pass at the same position does, for trees up to ``tail`` deep (the CPU path computes the
    same values without that rounding guarantee)."""
    scale = float(scale if scale is not None else q.shape[-1] ** -0.5)
    window = int(window or 0)
    _trace_attention(q, k_cache, mask, k_scale, keep, kivi, tail, softcap, sinks, window)
    if q.is_cuda:
        return require().attention(q, k_cache, v_cache, kv_len, n_new, mask, scale, int(q_offset), None, k_scale,
                                   v_scale, keep, lse_out, kivi, kivi_chunks, int(kivi_bits), int(tail),
                                   float(softcap or 0.0), sinks, window, pages)
    return reference.attention(q, k_cache, v_cache, kv_len, n_new, mask, scale, softcap=softcap, q_offset=q_offset,
                               k_scale=k_scale, v_scale=v_scale, keep=keep, lse_out=lse_out, kivi=kivi,
                               kivi_chunks=kivi_chunks, kivi_bits=kivi_bits, sinks=sinks, window=window, pages=pages)


_ATTENTION_USAGE: dict[tuple[str, str, int, str], int] = {}


def _trace_attention(q, k_cache, mask, k_scale, keep, kivi, tail, softcap=None, sinks=None, window=0) -> None:
    device = "cuda" if q.is_cuda else "cpu"
    cache = "kivi" if kivi is not None else "fp8" if k_scale is not None else str(k_cache.dtype).removeprefix("torch.")
    parts = ["masked" if mask is not None else "causal"]
    if tail:
        parts.append("exact_tail")
    if keep is not None:
        parts.append("keep")
    if softcap:
        parts.append("softcap")
    if sinks is not None:
        parts.append("sinks")
    if window:
        parts.append("window")
    key = (device, cache, int(q.shape[1]), "+".join(parts))
    _ATTENTION_USAGE[key] = _ATTENTION_USAGE.get(key, 0) + 1


def attention_usage(reset: bool = False) -> dict[tuple[str, str, int, str], int]:
    """Which attention paths ran: ``{(device, cache format, queries per row, mode): calls}``, counted when a call
    is issued from Python (a captured CUDA graph counts its calls once, at capture). The tracing economize does in
    ``attention/interface.py`` (``kernel_usage``)."""
    usage = dict(_ATTENTION_USAGE)
    if reset:
        _ATTENTION_USAGE.clear()
    return usage


def kivi_quantize(cache: torch.Tensor, kivi: torch.Tensor, kv_len: torch.Tensor, chunks: torch.Tensor, bits: int,
                  residual: int, max_new: int, pages: torch.Tensor | None = None) -> None:
    """Code newly committed 128-key chunks of every layer into KIVI storage and advance ``chunks`` (in place);
    ``pages [L, B, C]``: ``cache`` is a page pool ``[P, 2, H_kv, 128, D]``."""
    if cache.is_cuda:
        require().kivi_quantize(cache, kivi, kv_len, chunks, int(bits), int(residual), int(max_new), pages)
        return
    reference.kivi_quantize(cache, kivi, kv_len, chunks, bits, residual, max_new, pages)


def attention_scores(q: torch.Tensor, k_cache: torch.Tensor, kv_len: torch.Tensor, n_new: torch.Tensor,
                     mask: torch.Tensor | None, lse2: torch.Tensor, scores: torch.Tensor,
                     scale: float | None = None, q_offset: int = 0, pages: torch.Tensor | None = None) -> None:
    """Accumulate KV-eviction scores (H2O / SnapKV) into ``scores [B, H_kv, S]`` on the tensor cores."""
    scale = float(scale if scale is not None else q.shape[-1] ** -0.5)
    if q.is_cuda:
        require().attention_scores(q, k_cache, kv_len, n_new, mask, lse2, scores, scale, int(q_offset), pages)
        return
    reference.attention_scores(q, k_cache, kv_len, n_new, mask, lse2, scores, scale, q_offset, pages)


def silu_mul(gate_up: torch.Tensor | Partials) -> torch.Tensor:
    if gate_up.is_cuda:
        return require().silu_mul(_raw(gate_up))
    return reference.silu_mul(gate_up)


def gelu_tanh_mul(gate_up: torch.Tensor | Partials) -> torch.Tensor:
    """``gelu_tanh(gate) * up`` of a fused ``[gate; up]`` projection (GeGLU)."""
    if gate_up.is_cuda:
        return require().glu(_raw(gate_up), 1)
    return reference.gelu_tanh_mul(gate_up.sum() if isinstance(gate_up, Partials) else gate_up)


_GLU_ACTS = {"silu": 0, "gelu_tanh": 1, "clamped_swiglu": 2}


def vs_keep(cols: torch.Tensor, offsets: torch.Tensor, base: int, t: int, limit: int, size: int) -> torch.Tensor:
    """MInference's vertical-slash pattern of a query chunk (``t`` queries from position ``base``) as keep bit words
    ``int32 [..., size / 32]`` for the attention kernel: key columns ``cols [..., nv]`` and the keys that the slash
    diagonals ``offsets [..., ns]`` cross, below ``limit``. On CUDA ``csrc/minference.cu:vs_keep_kernel``."""
    if cols.is_cuda:
        return require().vs_keep(cols.long(), offsets.long(), base, t, limit, size)
    return reference.vs_keep(cols.long(), offsets.long(), base, t, limit, size)


def hadamard(x: torch.Tensor, block: int) -> torch.Tensor:
    """``x H_b / sqrt(b)`` over consecutive blocks of ``block`` (a power of two) of the last dimension: QuaRot's
    online rotation. On CUDA (bf16, ``8 <= block <= 8192``) the kernel of ``csrc/elementwise.cu:hadamard_kernel``."""
    if x.is_cuda and x.dtype == torch.bfloat16:
        return require().hadamard(x, block)
    return reference.hadamard(x, block)


def glu(gate_up: torch.Tensor | Partials, act: str = "silu", limit: float = 7.0, hadamard: int = 0) -> torch.Tensor:
    """The gated MLP activation ``act(gate) * up`` (``"silu"``: SwiGLU, ``"gelu_tanh"``: GeGLU,
    ``"clamped_swiglu"``: gpt-oss's ``(clamp(up, +-limit) + 1) * g * sigmoid(1.702 g)`` with ``g = min(gate,
    limit)``). ``hadamard > 0`` rotates the result by the block Hadamard transform of that block size in the same
    kernel (on CUDA), the online input rotation of a rotated down projection."""
    if hadamard:
        if act not in _GLU_ACTS:
            raise ValueError(f"unsupported gated activation {act!r}")
        if gate_up.is_cuda and (isinstance(gate_up, Partials) or gate_up.dtype == torch.bfloat16):
            return require().glu_hadamard(_raw(gate_up), _GLU_ACTS[act], limit, hadamard)
        dense = gate_up.sum() if isinstance(gate_up, Partials) else gate_up
        return reference.hadamard(reference.glu(dense, act, limit), hadamard)
    if act == "silu":
        return silu_mul(gate_up)
    if act == "gelu_tanh":
        return gelu_tanh_mul(gate_up)
    if act == "clamped_swiglu":
        if gate_up.is_cuda:
            return require().glu(_raw(gate_up), 2, limit)
        return reference.clamped_swiglu(gate_up.sum() if isinstance(gate_up, Partials) else gate_up, limit)
    raise ValueError(f"unsupported gated activation {act!r}")


def linear(x: torch.Tensor, weight, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ weight.T (+ bias)``; on CUDA the tcgen05/TMA GEMM of ``csrc/gemm_tc.cu``, or for a quantized
    :class:`~economize_b200.ops.quant.QWeight` the weight-only GEMM of ``csrc/gemm_wq.cu``."""
    if isinstance(weight, (QWeight, FP8BlockWeight, Sparse24Weight)) or hasattr(weight, "linear"):
        y = weight.linear(x)
        return y if bias is None else y + bias
    if x.is_cuda:
        shape = x.shape
        y = require().linear(x.reshape(-1, shape[-1]), weight)
        y = y.reshape(*shape[:-1], weight.shape[0])
        return y if bias is None else y + bias
    return reference.linear(x, weight, bias)


def argmax(x: torch.Tensor) -> torch.Tensor:
    """Index of the largest entry of every row of ``x [..., V]`` (first one on ties), as int64."""
    if x.is_cuda:
        shape = x.shape
        return require().argmax(x.reshape(-1, shape[-1])).reshape(shape[:-1])
    return x.argmax(-1)


def greedy_accept(tokens: torch.Tensor, parents: torch.Tensor, pred: torch.Tensor,
                  ok: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Longest accepted path of a verified chain or tree (see :func:`.reference.greedy_accept`)."""
    if tokens.is_cuda:
        return require().greedy_accept(tokens, parents, pred, ok)
    return reference.greedy_accept(tokens, parents, pred, ok)


def kv_compact(cache: torch.Tensor, kv_len: torch.Tensor, path: torch.Tensor, n_acc: torch.Tensor,
               pages: torch.Tensor | None = None) -> None:
    """Move an accepted path's cache entries to consecutive slots in every layer (in place); ``pages [L, B, C]``:
    ``cache`` is a page pool ``[P, 2, H_kv, 128, D]``."""
    if cache.is_cuda:
        require().kv_compact(cache, kv_len, path, n_acc, pages)
        return
    reference.kv_compact(cache, kv_len, path, n_acc, pages)


def sample(probs: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """One token per row of ``probs [..., V]`` (fp32) by inverse CDF at the uniforms ``u [...]``."""
    if probs.is_cuda:
        shape = probs.shape[:-1]
        return require().sample(probs.reshape(-1, probs.shape[-1]).float(), u.reshape(-1).float()).reshape(shape)
    return reference.sample(probs, u)


def rejection(p: torch.Tensor, q: torch.Tensor, drafts: torch.Tensor, u_acc: torch.Tensor,
              u_draw: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Lossless speculative sampling of draft chains: accept/reject every draft and draw the correction or bonus
    token in one kernel (see :func:`.reference.rejection`)."""
    if p.is_cuda:
        return require().rejection(p.float(), q.float(), drafts, u_acc.float(), u_draw.float())
    return reference.rejection(p, q, drafts, u_acc, u_draw)


def ngram(history: torch.Tensor, length: torch.Tensor, k: int, min_n: int, max_n: int,
          earliest: bool = True) -> torch.Tensor:
    """Prompt-lookup draft proposals ``[B, k]`` from the token history (see :func:`.reference.ngram`)."""
    if history.is_cuda:
        return require().ngram(history, length.to(torch.int32), int(k), int(min_n), int(max_n), bool(earliest))
    return reference.ngram(history, length, k, min_n, max_n, earliest)


def tree_layout(parents: torch.Tensor, kv_len: torch.Tensor, max_depth: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Ancestor bits ``[B, T]`` (int64) and positions ``kv_len + depth`` ``[B, T]`` (int32) of a verified tree given
    by ``parents [B, T]`` (root at node 0, ``parents[:, i] < i``); one kernel on CUDA."""
    if parents.is_cuda:
        return require().tree_layout(parents.long(), kv_len.int())
    from ..decoding.tree import ancestor_bits, popcount64

    bits = ancestor_bits(parents, max_depth)
    return bits, (kv_len[:, None] + (popcount64(bits) - 1)).to(torch.int32)


def topk_logp(logits: torch.Tensor, k: int, floor: float, d2t: torch.Tensor | None = None
              ) -> tuple[torch.Tensor, torch.Tensor]:
    """``k`` largest log-probabilities of every row of ``logits [..., V]`` (clamped below at ``floor``; ties: lower
    index) and their indices, mapped to target ids by ``index + d2t[index]`` when ``d2t`` is given."""
    if logits.is_cuda:
        return require().topk_logp(logits.float(), int(k), float(floor), d2t)
    logp = torch.log_softmax(logits.float(), -1).clamp_min(floor)
    top = logp.topk(k, -1)
    idx = top.indices
    return top.values, (idx + d2t[idx] if d2t is not None else idx)
