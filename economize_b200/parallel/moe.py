"""Sparse mixture-of-experts MLP (Mixtral-style top-k routing) on one GPU and with expert parallelism.

One GPU (:func:`moe_mlp`): router GEMM -> ``moe_route`` (softmax, top-k, renormalised weights, expert-ordered
positions) -> ``moe_gather`` -> grouped gate/up GEMM over all experts -> SwiGLU -> grouped down GEMM ->
``moe_combine``; all on the device, no host synchronisation, so MoE decode steps record into CUDA graphs. The
reference runs Hugging Face's MoE blocks (a Python loop over experts with a host-side ``nonzero`` per expert).

Expert parallelism (:class:`ExpertParallel`): rank ``r`` of ``P`` owns experts ``[r E/P, (r+1) E/P)`` and every
rank routes its own tokens. Dispatch and combine are all-to-all exchanges of the routed rows (``all_to_all_single``
of the per-rank counts, then of the rows and their local expert ids; NCCL on GPUs, Gloo on the CPU); the rows a
rank receives run through its experts and go back the same way, and the source rank sums each token's weighted
expert outputs in fp32.

Fused expert parallelism (:class:`FusedExpertParallel`): the same ownership, with the exchanges done by kernels
(``csrc/ep.cu``) that store the routed rows straight into the peers' IPC-mapped buffers over NVLink and signal with
system-scope counters. One MoE call is route -> gather -> dispatch -> segments -> grouped gate/up GEMM -> SwiGLU ->
grouped down GEMM -> combine -> weighted sum, all on the device without a host synchronisation, so expert-parallel
decode steps record into CUDA graphs. Economize runs MoE models through Hugging Face's blocks only (no expert
parallelism of its own).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .. import ops
from ..errors import CommTimeoutError, ConfigError
from ..ops import reference

__all__ = ["ExpertParallel", "FusedExpertParallel", "moe_mlp", "moe_reference", "route", "shard_experts"]


def route(logits: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Top-``k`` experts per row and their weights renormalised over the chosen ones (fp32; ties: lower id)."""
    probs = torch.softmax(logits.float(), -1)
    w, ids = torch.topk(probs, k, dim=-1, sorted=True)
    return ids, w / w.sum(-1, keepdim=True)


def moe_reference(x: torch.Tensor, router: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor,
                  k: int, renormalize: bool = True, logits: torch.Tensor | None = None, act: str = "silu",
                  limit: float = 7.0, biases: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None
                  ) -> torch.Tensor:
    """The MoE MLP in plain PyTorch (fp32 accumulation of the weighted expert outputs); ``logits`` overrides the
    router output (to route exactly like another implementation). ``act``: the gated activation of
    :func:`economize_b200.ops.glu`; ``biases``: (router [E], gate/up [E, 2F], down [E, H]) of gpt-oss experts."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    b_router, b_gate_up, b_down = biases if biases is not None else (None, None, None)
    scores = F.linear(x2, router, b_router) if logits is None else logits
    ids, w = route(scores, k)
    if not renormalize:
        w = w * torch.softmax(scores.float(), -1).gather(-1, ids).sum(-1, keepdim=True).to(w.dtype)
    out = torch.zeros(x2.shape[0], shape[-1], dtype=torch.float32, device=x.device)
    for e in range(w_gate_up.shape[0]):
        rows, slot = (ids == e).nonzero(as_tuple=True)
        if rows.numel() == 0:
            continue
        gu = F.linear(x2[rows], w_gate_up[e], None if b_gate_up is None else b_gate_up[e])
        y = F.linear(reference.glu(gu, act, limit), w_down[e], None if b_down is None else b_down[e])
        out.index_add_(0, rows, y.float() * w[rows, slot][:, None])
    return out.to(x.dtype).reshape(shape)


def _expert_rows(offsets: torch.Tensor, rows: int) -> torch.Tensor:
    """The expert of every expert-ordered row (``offsets [E + 1]``), found on the device without a host sync."""
    return torch.searchsorted(offsets[1:].contiguous(), torch.arange(rows, device=offsets.device, dtype=torch.int32),
                              right=True)


def moe_mlp(x: torch.Tensor, router: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor,
            k: int, ep: ExpertParallel | None = None, renormalize: bool = True, act: str = "silu",
            limit: float = 7.0, biases: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None
            ) -> torch.Tensor:
    """Top-``k`` MoE MLP of ``x [..., H]`` with experts ``w_gate_up [E, 2F, H]``, ``w_down [E, H, F]``. The
    chosen experts' softmax probabilities are renormalised to sum to one (Mixtral; for gpt-oss this is its softmax
    over the top-k logits), or kept as they are (``renormalize=False``, Qwen3-MoE's ``norm_topk_prob=False``).
    ``act`` is the experts' gated activation and ``biases`` the gpt-oss router and expert biases (router [E],
    gate/up [E, 2F], down [E, H]): on the GPU each grouped GEMM's rows get their expert's bias before the
    activation and before the weighted combine."""
    if ep is not None and ep.size > 1:
        if not renormalize:
            raise ConfigError("expert parallelism renormalises the top-k router weights")
        if act != "silu" or biases is not None:
            raise ConfigError("expert parallelism runs SwiGLU experts without biases")
        return ep.forward(x, router, w_gate_up, w_down, k)
    if not x.is_cuda:
        return moe_reference(x, router, w_gate_up, w_down, k, renormalize, act=act, limit=limit, biases=biases)
    from ..ops._ext import require

    C = require()
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).contiguous()
    logits = ops.linear(x2, router, None if biases is None else biases[0])
    ids, weights, pos, offsets = C.moe_route(logits, k)
    if not renormalize:  # back from the renormalised weights to the softmax probabilities of the chosen experts
        chosen = torch.softmax(logits.float(), -1).gather(-1, ids.long()).sum(-1, keepdim=True)
        weights = weights * chosen
    xs = C.moe_gather(x2, pos)
    gu = C.linear_grouped(xs, w_gate_up, offsets)
    if biases is not None:
        expert = _expert_rows(offsets, gu.shape[0])
        gu = gu + biases[1].index_select(0, expert)
    a = ops.glu(gu, act, limit)
    y = C.linear_grouped(a, w_down, offsets)
    if biases is not None:
        y = y + biases[2].index_select(0, expert)
    return C.moe_combine(y, pos, weights).reshape(shape)


class ExpertParallel:
    """Expert-parallel execution of a MoE layer over a process group (ranks own contiguous expert blocks).

    Args:
        rank, size: This rank and the group size.
        group: The process group (NCCL on GPUs, Gloo on the CPU).
    """

    def __init__(self, rank: int, size: int, group=None) -> None:
        self.rank, self.size, self.group = rank, size, group

    def owned(self, num_experts: int) -> range:
        if num_experts % self.size:
            raise ConfigError(f"{num_experts} experts do not split over {self.size} ranks")
        per = num_experts // self.size
        return range(self.rank * per, (self.rank + 1) * per)

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int]) -> None:
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, x: torch.Tensor, router: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor,
                k: int) -> torch.Tensor:
        """``w_gate_up``/``w_down`` hold this rank's experts only (``[E/P, 2F, H]``, ``[E/P, H, F]``); ``router``
        covers all ``E`` experts."""
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        T, H = x2.shape
        E = router.shape[0]
        per = E // self.size
        ids, w = route(ops.linear(x2, router), k)
        flat = ids.reshape(-1)
        order = torch.argsort(flat * (T * k) + torch.arange(T * k, device=x.device), stable=True)
        dest = (flat // per)[order]
        send_counts = torch.bincount(dest, minlength=self.size)
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, [1] * self.size, [1] * self.size)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        rows = x2[order // k]
        local_ids = (flat[order] - dest * per).to(torch.int64)
        recv = torch.empty(sum(rc), H, dtype=x.dtype, device=x.device)
        recv_ids = torch.empty(sum(rc), dtype=torch.int64, device=x.device)
        self._a2a(recv, rows.contiguous(), rc, sc)
        self._a2a(recv_ids, local_ids.contiguous(), rc, sc)
        y = torch.empty_like(recv)
        if recv.is_cuda and recv.shape[0]:  # this rank's experts as one grouped GEMM pair on the tensor cores
            from ..ops._ext import require

            C = require()
            by_expert = torch.argsort(recv_ids, stable=True)
            counts = torch.zeros(per, dtype=torch.int64, device=x.device).index_add_(
                0, recv_ids, torch.ones_like(recv_ids))
            offsets = torch.cat([counts.new_zeros(1), counts.cumsum(0)]).to(torch.int32)
            a = ops.silu_mul(C.linear_grouped(recv[by_expert].contiguous(), w_gate_up, offsets))
            y[by_expert] = C.linear_grouped(a, w_down, offsets)
        else:
            for e in range(per):  # experts of this rank
                sel = (recv_ids == e).nonzero(as_tuple=True)[0]
                if sel.numel() == 0:
                    continue
                g, u = F.linear(recv[sel], w_gate_up[e]).chunk(2, -1)
                y[sel] = F.linear(F.silu(g) * u, w_down[e])
        back = torch.empty_like(rows)
        self._a2a(back, y, sc, rc)
        out = torch.zeros(T, H, dtype=torch.float32, device=x.device)
        weight = w.reshape(-1)[order]
        out.index_add_(0, order // k, back.float() * weight[:, None])
        return out.to(x.dtype).reshape(shape)


class FusedExpertParallel(ExpertParallel):
    """Expert parallelism whose dispatch and combine are peer stores over NVLink (no NCCL call per MoE layer).

    Every rank allocates one symmetric buffer (received rows, their source rows, per-expert counts, returned rows
    and the arrival counters) and maps every peer's through CUDA IPC; the handles travel once through
    ``torch.distributed``. Calls with more than ``max_tokens`` tokens use the all-to-all path of
    :class:`ExpertParallel`, so every rank must see the same side of that bound in a call (lockstep decoding with
    equal batches does). Ranks must share a node with NVLink peer access.

    Args:
        rank, size, group: As for :class:`ExpertParallel`.
        max_tokens: Most tokens one rank routes in one fused call (sizes the buffers: every rank may send all its
            ``max_tokens * k`` rows to one peer).
    """

    def __init__(self, rank: int, size: int, group=None, max_tokens: int = 256) -> None:
        super().__init__(rank, size, group)
        if size > 8:
            raise ConfigError("the fused expert-parallel exchange supports up to 8 ranks")
        self.max_tokens = max_tokens
        self._ext = None
        self._own = 0
        self.ptrs: list[int] = []
        self._shape: tuple[int, int, int] | None = None

    def setup(self, hidden: int, experts_local: int, k: int) -> None:
        """Allocate and map the buffers for MoE layers of width ``hidden`` with ``experts_local`` experts per rank
        and top-``k`` routing (collective: every rank calls it)."""
        if self._shape == (hidden, experts_local, k):
            return
        if self.size * experts_local > 128:
            raise ConfigError("the fused exchange supports at most 128 (rank, expert) pairs")
        self.close()
        ext = ops.require()
        self._ext = ext
        self.cap = self.max_tokens * k
        nbytes = ext.ep_buffer_bytes(self.size, experts_local, self.cap, hidden, self.cap)
        self._own, handle = ext.symm_alloc(nbytes)
        handles: list = [None] * self.size
        dist.all_gather_object(handles, handle, group=self.group)
        self.ptrs = [self._own if r == self.rank else ext.symm_open(h) for r, h in enumerate(handles)]
        dist.barrier(group=self.group)
        self._shape = (hidden, experts_local, k)

    def forward(self, x: torch.Tensor, router: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor,
                k: int) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        T, H = x2.shape
        if (not x.is_cuda or T > self.max_tokens or self._shape != (H, w_gate_up.shape[0], k)):
            return super().forward(x, router, w_gate_up, w_down, k)
        C = self._ext
        logits = ops.linear(x2, router)
        _, weights, pos, offsets = C.moe_route(logits, k)
        xs = C.moe_gather(x2, pos)
        out = C.ep_moe(xs, offsets, pos, weights, w_gate_up, w_down, self.ptrs, self.rank, self.cap, self.cap)
        return out.reshape(shape)

    def check(self) -> None:
        """Raise :class:`CommTimeoutError` if a bounded wait of this device gave up since the last check."""
        status = self._ext.status(torch.cuda.current_device()) if self._ext is not None else 0
        if status & 8:
            raise CommTimeoutError(f"a peer's expert rows did not arrive in time (status {status})")

    def close(self) -> None:
        if self._ext is None or not self.ptrs:
            return
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                self._ext.symm_close(p)
        self._ext.symm_free(self._own)
        self.ptrs, self._shape = [], None


def shard_experts(model, ep: ExpertParallel) -> None:
    """Keep this rank's experts in every MoE layer of an engine model and attach ``ep``."""
    with torch.no_grad():
        for layer in model.layers:
            if layer.router is None:
                continue
            own = ep.owned(layer.router.shape[0])
            layer.w_gate_up = torch.nn.Parameter(layer.w_gate_up.data[own.start:own.stop].contiguous())
            layer.w_down = torch.nn.Parameter(layer.w_down.data[own.start:own.stop].contiguous())
            if isinstance(ep, FusedExpertParallel) and layer.w_gate_up.is_cuda:
                ep.setup(layer.w_down.shape[1], len(own), model.config.experts_per_token)
    model.ep = ep
