"""The speculative-decoding engine: a device-resident cycle recorded as one CUDA graph.

economize's ``CycleDecoder`` (``src/economize/decoding/loop.py:57-258``) runs a cycle as Python over Hugging Face
layers and reads the accepted counts back to the host after every verification (``decoding/commit.py:37-75``); its
tree verifier loops over nodes on the host (``decoding/verifiers.py:139-158``). Here every step of a cycle is a
fixed-shape device computation, so the whole cycle is captured once per batch size and replayed:

    draft     root logits -> top-k -> (depth-1) batched tree steps of the drafter -> best ``total_tokens``
    verify    one target pass over root + tree with 64-bit ancestor masks (tree attention kernel)
    accept    argmax of the target logits -> longest accepted path (greedy_accept kernel)
    commit    KV of the accepted path moved to consecutive slots in every layer (kv_compact kernel),
              tokens appended to the output buffer, lengths advanced
    observe   the drafter's state for the committed columns + the next root step

The host only polls the generated lengths, every ``n`` cycles where ``n`` is the number of cycles that cannot
finish any row yet, so no cycle waits on the host.
"""

from __future__ import annotations

import functools
import math
from dataclasses import dataclass, field

import torch

from .. import ops
from ..errors import ConfigError
from ..models.llama import CausalLM
from ..runtime.cache import KVCache, PagedKVCache, StepBatch
from ..runtime.phase import phase
from .config import DecodeConfig
from .drafter import DraftModel
from .kv_stats import held_bytes, keep_snapshot, row_kv_stats
from .policies import POLICIES, ConfidencePolicy, DynamicTreePolicy, SequoiaPolicy, SpecExecPolicy
from .sequoia import AcceptanceProfile, StaticPlan, StaticTree, record_cycle
from .specexec import SearchOptions
from .tree import LOGP_FLOOR, TreeOptions, select_candidates
from .verifiers import VERIFIERS, RejectionVerifier, TypicalVerifier

__all__ = ["DecodeResult", "GenerationStats", "SpecEngine"]


@dataclass
class DecodeResult:
    """Generated tokens of one row and how they were produced.

    Attributes:
        tokens: The generated tokens (prompt excluded), truncated at ``max_new_tokens`` and at a stop token.
        cycles: Exact (verification) passes the row took after the prefill.
        accepted: Draft tokens accepted over those passes.
    """

    tokens: torch.Tensor
    cycles: int = 0
    accepted: int = 0
    #: every model call of the generation (:class:`~economize_b200.decoding.cost.CostLog`), when recorded
    cost: object = None
    #: computes the row's KV memory accounting on first access (see :attr:`kv`)
    _kv_source: object = field(default=None, repr=False, compare=False)
    _kv: object = field(default=None, repr=False, compare=False)

    @property
    def kv(self):
        """KV-cache bytes of the row (:class:`~economize_b200.decoding.kv_stats.RowKVStats`: stored and full-format
        committed bytes at the last pass, and the bytes attention read summed over the passes)."""
        if self._kv is None and self._kv_source is not None:
            self._kv = self._kv_source()
        return self._kv

    @property
    def mean_accepted(self) -> float:
        """Accepted drafts per verified cycle (economize's ``DecodeResult.mean_accepted``)."""
        return self.accepted / self.cycles if self.cycles else 0.0

    @property
    def mean_accepted_length(self) -> float:
        """Tokens committed per exact pass: ``1 + accepted drafts / passes`` (the paper's tau)."""
        return 1.0 + self.mean_accepted

    def cost_summary(self) -> dict[str, float]:
        return {"exact_passes": float(self.cycles), "accepted_drafts": float(self.accepted),
                "mean_accepted_length": self.mean_accepted_length, "new_tokens": float(self.tokens.numel())}


@dataclass
class GenerationStats:
    cycles: int = 0
    graph_replays: int = 0
    host_syncs: int = 0
    #: measured bytes of the last generation's KV buffers (cache, KIVI codes, keep bitmaps)
    kv_allocated_bytes: int = 0
    rows: list[DecodeResult] = field(default_factory=list)

    @property
    def mean_accepted_length(self) -> float:
        c = sum(r.cycles for r in self.rows)
        a = sum(r.accepted for r in self.rows)
        return 1.0 + a / c if c else 1.0


class _State:
    """Persistent device buffers of one (batch, capacity) configuration (graph inputs and outputs)."""

    def __init__(self, model: CausalLM, drafter: DraftModel | None, batch: int, capacity: int, out_cap: int,
                 draft_vocab: int, layout: dict | None = None) -> None:
        dev = model.device
        self.batch, self.capacity, self.out_cap = batch, capacity, out_cap
        self.cache: KVCache | PagedKVCache = model.new_cache(batch, capacity, **(layout or {}))
        i32 = dict(dtype=torch.int32, device=dev)
        self.kv_len = torch.zeros(batch, **i32)
        self.last = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.out = torch.zeros(batch, out_cap + 1, dtype=torch.int64, device=dev)  # last column: trash
        self.n_out = torch.zeros(batch, **i32)
        self.max_new = torch.zeros(batch, **i32)
        self.accepted = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.cycles = torch.zeros(batch, **i32)
        # drafts accepted by each row's cycles, in order (column out_cap: a trash slot); read back for the cost log
        self.acc_hist = torch.zeros(batch, out_cap + 1, **i32)
        # prompt + committed tokens + the pending root, slot p = position p (read by n-gram drafters)
        self.history = torch.zeros(batch, capacity + 1, dtype=torch.int64, device=dev)
        hidden = model.config.hidden_size
        if drafter is not None:
            self.carry = torch.zeros(batch, max(drafter.carry_size, 1), dtype=model.dtype, device=dev)
            self.root_logits = torch.zeros(batch, draft_vocab, dtype=torch.float32, device=dev)
            self.root_state = torch.zeros(batch, hidden, dtype=model.dtype, device=dev)


class SpecEngine:
    """Generates with a target :class:`~economize_b200.models.CausalLM` and an optional drafter.

    Args:
        model: The target model.
        drafter: The drafting technique's device-side drafter (``None``: plain decoding).
        config: Decoding options; ``cycle_length`` drafts per cycle (chains) or ``draft_policy="dynamic_tree"``.
        draft_vocab: Size of the drafter's vocabulary (for its logits buffer).
    """

    def __init__(self, model: CausalLM, drafter: DraftModel | None, config: DecodeConfig,
                 draft_vocab: int | None = None, selector=None) -> None:
        self.model = model
        self.config = config
        self.drafter = drafter if config.cycle_length > 1 else None
        self.draft_vocab = draft_vocab or model.config.vocab_size
        self.selector = selector if selector is not None and not getattr(selector, "greedy", True) else None
        self.verifier = VERIFIERS.get(config.verifier_name)(config)
        self.policy = POLICIES.get(config.draft_policy_name)(config)
        self.accept_all = config.verifier_name == "accept_all"
        self.tree: TreeOptions | None = None  # EAGLE-2 dynamic trees
        self.static_tree: StaticTree | None = None  # Sequoia
        self.search: SearchOptions | None = None  # SpecExec
        self.acceptance: AcceptanceProfile | None = None
        self._plans: dict[torch.device, StaticPlan] = {}
        if self.drafter is not None and self.policy.drafts_tree:
            if not self.verifier.supports_trees or self.verifier.needs_draft_probs:
                raise ConfigError(f"draft_policy {config.draft_policy_name!r} drafts trees, which verifier "
                                  f"{config.verifier_name!r} cannot verify; use greedy or typical")
            if isinstance(self.policy, DynamicTreePolicy):
                self.tree = self.policy.options
            else:
                if hasattr(self.drafter, "propose"):
                    raise ConfigError(f"draft_policy {config.draft_policy_name!r} needs a drafter with tree steps; "
                                      f"{type(self.drafter).__name__} proposes its own drafts")
                if isinstance(self.policy, SequoiaPolicy):
                    self.static_tree = self.policy.tree
                    self.acceptance = AcceptanceProfile() if self.policy.record else None
                elif isinstance(self.policy, SpecExecPolicy):
                    self.search = self.policy.options
        self.rejection = isinstance(self.verifier, RejectionVerifier) and self.selector is not None
        self.min_confidence = self.policy.min_confidence if isinstance(self.policy, ConfidencePolicy) else None
        self.static = self.drafter is not None and hasattr(self.drafter, "propose")
        if self.drafter is None:
            self.depth = 0
            self.nodes = 0
        elif self.static:
            self.tree = None
            self.depth = self.drafter.draft_depth(config)
            self.nodes = self.drafter.draft_nodes(config)
        elif self.tree is not None:
            self.depth = self.tree.depth
            self.nodes = self.tree.total_tokens
        elif self.static_tree is not None:
            self.depth = self.static_tree.depth
            self.nodes = self.static_tree.size
        elif self.search is not None:
            self.depth = self.search.depth
            self.nodes = self.search.total_tokens
        else:
            self.depth = config.cycle_length - 1
            self.nodes = self.depth
        shape = self.tree or self.static_tree or self.search
        self.forwarded = shape.forwarded if shape is not None else self.depth
        self._states: dict[tuple[int, int, int], _State] = {}
        self._graphs: dict[tuple[int, int, int], torch.cuda.CUDAGraph] = {}
        self.stats = GenerationStats()

    # ---- public ------------------------------------------------------------------------------------------------
    @property
    def tokens_per_cycle(self) -> int:
        return self.depth + 1

    def capacity_for(self, prompt_len: int, max_new: int) -> int:
        slack = self.nodes + 2 + self.depth + self.forwarded + 8
        return int(math.ceil((prompt_len + max_new + slack) / 128) * 128)

    @torch.no_grad()
    def generate(self, prompts: list[torch.Tensor] | torch.Tensor, max_new_tokens: int | list[int],
                 stop_tokens: list[int] | None = None) -> list[DecodeResult]:
        """Generate after every prompt (1-D tensors of any length, or the rows of a ``[B, P]`` tensor)."""
        if isinstance(prompts, torch.Tensor):
            prompts = list(prompts) if prompts.dim() == 2 else [prompts]
        batch = len(prompts)
        max_news = [max_new_tokens] * batch if isinstance(max_new_tokens, int) else list(max_new_tokens)
        longest = max(p.numel() for p in prompts)
        max_new = max(max_news)
        capacity = self.capacity_for(longest, max_new)
        out_cap = max_new + self.depth + 2
        state = self._state(batch, capacity, out_cap)
        dev = self.model.device
        lengths = torch.tensor([p.numel() for p in prompts], dtype=torch.int32)
        padded = torch.zeros(batch, longest, dtype=torch.int64)
        for i, p in enumerate(prompts):
            padded[i, : p.numel()] = p.reshape(-1).cpu()
        self._prefill(state, padded.to(dev, non_blocking=True), lengths.to(dev, non_blocking=True),
                      torch.tensor(max_news, dtype=torch.int32).to(dev, non_blocking=True))
        self._run_cycles(state, max_new, stop_tokens)
        n_out = state.n_out.cpu()
        out = state.out[:, :out_cap].cpu()
        acc = state.accepted.cpu()
        cyc = state.cycles.cpu()
        hist = state.acc_hist.cpu() if self.drafter is not None else None
        results = []
        keep = keep_snapshot(self.model)
        for b in range(batch):
            toks = out[b, : min(int(n_out[b]), max_news[b])]
            if stop_tokens:
                hits = [i for i, t in enumerate(toks.tolist()) if t in stop_tokens]
                if hits:
                    toks = toks[: hits[0] + 1]
            accepted = hist[b, : int(cyc[b])].tolist() if hist is not None else [0] * int(cyc[b])
            res = DecodeResult(toks, int(cyc[b]), int(acc[b]), self.cost_log(int(lengths[b]), accepted))
            res._kv_source = functools.partial(row_kv_stats, self.model, keep, b, int(lengths[b]), accepted)
            results.append(res)
        self.stats.rows = results
        self.stats.kv_allocated_bytes = held_bytes(self.model, state.cache)
        return results

    # ---- cost accounting ---------------------------------------------------------------------------------------
    def _draft_footprint(self):
        from .cost import LayerFootprint

        drafter = self.drafter
        footprint = getattr(drafter, "footprint", None)
        if footprint is not None:
            return footprint() if callable(footprint) else footprint
        name = getattr(drafter, "cost_module", None) or type(drafter).__name__.removesuffix("Drafter").lower()
        return LayerFootprint.of(range(1, int(getattr(drafter, "num_layers", 1)) + 1), module=name)

    def _draft_steps(self) -> list[int]:
        """Tokens of each draft step of one cycle that runs a draft network (the first draft comes from the
        previous cycle's observe pass, so a chain of k drafts makes k - 1 calls)."""
        if self.drafter is None or self.static:
            return []
        if self.tree is not None:
            return [self.tree.topk] * (self.tree.depth - 1)
        if self.static_tree is not None:
            return list(self._plan(self.model.device).widths[:-1]) if self.static_tree.depth > 1 else []
        if self.search is not None:
            return [self.search.width] * (self.search.depth - 1)
        return [1] * (self.depth - 1)

    def cost_log(self, prompt_tokens: int, accepted: list[int]):
        """The model calls of one row: the prefill, then per cycle the draft steps, the verification pass over the
        draft tree and the drafter's observe pass, with ``accepted[c]`` drafts accepted by cycle ``c``."""
        from .cost import CostKind, CostLog, LayerFootprint

        log = CostLog()
        target = LayerFootprint.all(self.model.config.num_layers)
        log.record_footprint(CostKind.EXACT, prompt_tokens, 0, target)
        position = prompt_tokens
        if self.drafter is None:
            for _ in accepted:
                log.record_footprint(CostKind.EXACT, 1, position, target)
                position += 1
            return log
        draft = self._draft_footprint()
        steps = self._draft_steps()
        verified = 1 + (self.tree.total_tokens if self.tree is not None else
                        self.static_tree.size if self.static_tree is not None else
                        self.search.total_tokens if self.search is not None else
                        self.drafter.draft_nodes(self.config) if self.static else self.depth)
        observes = getattr(self.drafter, "observes", True) and not self.static
        for n_acc in accepted:
            for i, width in enumerate(steps):
                log.record_footprint(CostKind.DRAFT, width, position + i + 1, draft, step=i + 1)
            log.record_footprint(CostKind.EXACT, verified, position, target)
            if observes:
                log.record_footprint(CostKind.DRAFT_OBSERVE, n_acc + 2, position, draft)
            position += n_acc + 1
        return log

    # ---- state -------------------------------------------------------------------------------------------------
    @property
    def paged(self) -> bool:
        return bool(self.config.window_cache or self.config.kv_pages)

    def ring_reserve(self) -> int:
        """New slots one pass of this engine may write into a ring cache: a prefill chunk or a verification tree."""
        chunk = self.config.prefill_chunk or 512
        return int(math.ceil(max(chunk, self.nodes + self.depth + 2) / 128) * 128)

    def _layout(self) -> dict | None:
        if not self.paged:
            return None
        m = self.model
        if m.kv_evictor is not None or m.prefill_sparsity is not None:
            raise ConfigError("paged and ring caches do not serve keep-bitmap KV techniques (eviction, sparse "
                              "views); use the contiguous cache (window_cache=False, kv_pages=False)")
        return dict(paged=True, rings=self.config.window_cache, reserve=self.ring_reserve())

    def _state(self, batch: int, capacity: int, out_cap: int) -> _State:
        key = (batch, capacity, out_cap)
        st = self._states.get(key)
        if st is None:
            # one live configuration at a time keeps memory bounded; graphs of other shapes are dropped
            self._states = {k: v for k, v in self._states.items() if k[0] == batch}
            self._graphs = {k: v for k, v in self._graphs.items() if k in self._states}
            st = _State(self.model, self.drafter, batch, capacity, out_cap, self.draft_vocab, self._layout())
            self._states[key] = st
        else:
            st.cache.reset()
            st.n_out.zero_()
            st.accepted.zero_()
            st.cycles.zero_()
        if self.drafter is not None:
            self.drafter.begin(batch, capacity)
            if hasattr(self.drafter, "bind_target_cache"):  # drafters that run target layers (Hidden Transfer)
                self.drafter.bind_target_cache(st.cache)
        return st

    # ---- prefill -----------------------------------------------------------------------------------------------
    def _prefill(self, st: _State, prompts: torch.Tensor, lengths: torch.Tensor, max_new: torch.Tensor) -> None:
        model, drafter = self.model, self.drafter
        batch, width = prompts.shape
        capture = drafter.capture_layers if drafter is not None else ()
        chunk = self.config.prefill_chunk
        if self.config.window_cache and any(getattr(st.cache, "rings", ())):
            chunk = min(chunk or st.cache.reserve, st.cache.reserve)  # a pass may not lap a ring
        model.begin_sequence(st.cache)
        with phase("prefill"):
            if chunk is not None and width > chunk:
                hidden, aux = self._chunked_prefill(st, prompts, lengths, chunk, capture)
            else:
                hidden, aux = model.forward_step(prompts, StepBatch.prefill(lengths, width), st.cache, capture)
        last_idx = (lengths.long() - 1).clamp_min(0)
        rows = torch.arange(batch, device=prompts.device)
        bonus = self._pred(hidden[rows, last_idx])
        st.kv_len.copy_(lengths)
        model.after_commit(st.cache, st.kv_len, prefill=True)
        st.last.copy_(bonus)
        st.history.zero_()
        st.history[:, :width] = prompts
        st.history[rows, lengths.long()] = bonus
        st.out.zero_()
        st.out[:, 0] = bonus
        st.n_out.fill_(1)
        st.max_new.copy_(max_new)
        if drafter is not None and getattr(drafter, "observes", True):
            fused = drafter.fuse(aux)  # [B, P, d]
            tokens = torch.cat([prompts, torch.zeros_like(prompts[:, :1])], 1)
            tokens[rows, lengths.long()] = bonus
            sources = torch.cat([torch.zeros_like(fused[:, :1]), fused], 1)
            n_valid = lengths + 1
            with phase("draft"):
                root_logits, root_state = drafter.observe(tokens, sources, torch.zeros_like(lengths), n_valid,
                                                          lengths)
            if root_logits is not None:
                st.root_logits.copy_(root_logits)
                st.root_state.copy_(root_state)
            st.carry.copy_(fused[rows, last_idx])

    def _chunked_prefill(self, st: _State, prompts: torch.Tensor, lengths: torch.Tensor, chunk: int,
                         capture: tuple[int, ...]) -> tuple[torch.Tensor, dict[int, torch.Tensor]]:
        """Prefill in consecutive causal chunks (activations scale with the chunk, not the prompt)."""
        batch, width = prompts.shape
        hs, auxes = [], []
        for start in range(0, width, chunk):
            end = min(width, start + chunk)
            part = prompts[:, start:end]
            n = (lengths - start).clamp(0, end - start).to(torch.int32)
            kv = torch.clamp(lengths, max=start).to(torch.int32)
            pos = (start + torch.arange(end - start, device=prompts.device, dtype=torch.int32)).expand(batch, -1)
            h, a = self.model.forward_step(part, StepBatch(kv, n, pos.contiguous(), prompt=True), st.cache, capture)
            hs.append(h)
            auxes.append(a)
        hidden = torch.cat(hs, 1)
        aux = {k: torch.cat([a[k] for a in auxes], 1) for k in auxes[0]}
        return hidden, aux

    # ---- cycles ------------------------------------------------------------------------------------------------
    def _run_cycles(self, st: _State, max_new: int, stop_tokens: list[int] | None) -> None:
        # drafters that search host-side structures (retrieval, suffix trees) synchronise with the host every cycle
        use_graph = self.config.cuda_graphs and self.model.device.type == "cuda" and \
            getattr(self.drafter, "graph_safe", True) and self.acceptance is None and \
            getattr(self.model, "placement", None) is None  # a graph belongs to one device
        key = (st.batch, st.capacity, st.out_cap)
        remaining = max_new - 1  # the prefill produced the first token
        per_cycle = self.tokens_per_cycle
        while remaining > 0:
            # cycles that cannot finish any row even if every draft is accepted
            n = max(1, math.ceil(remaining / per_cycle))
            for _ in range(n):
                if use_graph:
                    graph = self._graphs.get(key)
                    if graph is None:
                        self._cycle(st)  # warm-up cycles run eagerly and produce real tokens
                        self._cycle(st)
                        graph = self._capture(st)
                        self._graphs[key] = graph
                        self.stats.cycles += 2
                        continue
                    graph.replay()
                    self.stats.graph_replays += 1
                else:
                    self._cycle(st)
                self.stats.cycles += 1
            self.stats.host_syncs += 1
            done = st.n_out - st.max_new
            if stop_tokens:
                hit = torch.isin(st.out[:, : st.out_cap], torch.tensor(stop_tokens, device=st.out.device)).any(1)
                done = torch.where(hit, torch.zeros_like(done), done)
            remaining = int(-done.min().item())

    def _capture(self, st: _State) -> torch.cuda.CUDAGraph:
        graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph):
            self._cycle(st, capturing=True)
        return graph

    def _cycle(self, st: _State, capturing: bool = False) -> None:
        if self.drafter is None:
            self._plain_cycle(st)
        else:
            self._spec_cycle(st)
        self.model.after_commit(st.cache, st.kv_len)  # KV coders compress what became old (inside the graph)

    def _plain_cycle(self, st: _State) -> None:
        model = self.model
        batch = st.batch
        one = torch.ones(batch, dtype=torch.int32, device=st.kv_len.device)
        sb = StepBatch(st.kv_len, one, st.kv_len[:, None].contiguous(),
                       torch.ones(batch, 1, dtype=torch.int64, device=st.kv_len.device))
        with phase("decode"):
            hidden, _ = model.forward_step(st.last[:, None], sb, st.cache)
        pred = self._pred(hidden[:, 0])
        active = st.n_out < st.max_new
        st.out.scatter_(1, torch.where(active, st.n_out, st.out_cap).long()[:, None], pred[:, None])
        step = active.to(st.kv_len.dtype)
        st.n_out.add_(step)  # finished rows keep their output length and their KV position
        st.kv_len.add_(step)
        st.cycles.add_(active.int())
        st.last.copy_(pred)

    def _spec_cycle(self, st: _State) -> None:
        model, drafter = self.model, self.drafter
        batch, dev = st.batch, st.kv_len.device
        depth = self.depth
        q_full = None
        with phase("draft"):
            if self.static:
                draft_tokens, draft_parents = drafter.propose(st.history, st.kv_len + 1)
            elif self.tree is not None:
                draft_tokens, draft_parents = self._draft_tree(st)
            elif self.static_tree is not None:
                draft_tokens, draft_parents = self._draft_static_tree(st)
            elif self.search is not None:
                draft_tokens, draft_parents = self._draft_search(st)
            else:
                draft_tokens, draft_parents, q_full = self._draft_chain(st)
            overlay = getattr(drafter, "overlay", None)  # a hybrid lays its primary's proposals over the drafts
            if overlay is not None:
                draft_tokens, draft_parents, q_full = overlay(st.history, st.kv_len + 1, draft_tokens, draft_parents,
                                                              q_full)
        # ---- verify: root + drafts in one tree pass ----
        tokens = torch.cat([st.last[:, None], draft_tokens], 1)  # [B, T]
        length = tokens.shape[1]
        parents = torch.cat([torch.zeros(batch, 1, dtype=torch.int64, device=dev), draft_parents + 1], 1)
        bits, positions = ops.tree_layout(parents, st.kv_len, depth)
        n_new = torch.full((batch,), length, dtype=torch.int32, device=dev)
        sb = StepBatch(st.kv_len, n_new, positions, bits)
        with phase("refresh"):
            hidden, aux = model.forward_step(tokens.clamp_min(0), sb, st.cache, drafter.capture_layers)
        self.last_pred = None
        n_acc, path, out = self._verify(tokens, parents, hidden, draft_tokens, q_full)
        after = getattr(drafter, "after_verify", None)
        if after is not None:  # host-side drafters that read the pass's predictions at their own nodes
            after(tokens, self.last_pred)
        if self.acceptance is not None:  # Sequoia rate measurement: one host synchronization per cycle
            record_cycle(self.acceptance, self.static_tree, self._plan(dev), tokens, path, n_acc, out)
        st.cache.compact(st.kv_len, path, n_acc)
        # ---- commit ----
        active = st.n_out < st.max_new
        width = depth + 1
        col = torch.arange(width, device=dev)[None]
        idx = st.n_out.long()[:, None] + col
        keep = (col <= n_acc.long()[:, None]) & (idx < st.out_cap) & active[:, None]
        st.out.scatter_(1, torch.where(keep, idx, st.out_cap), out[:, :width])
        st.accepted.add_(torch.where(active, n_acc, 0).long())
        st.acc_hist.scatter_(1, torch.where(active, st.cycles, st.out_cap).long()[:, None], n_acc[:, None].int())
        st.cycles.add_(active.int())
        hist_idx = st.kv_len.long()[:, None] + 1 + col
        hist_keep = (col <= n_acc.long()[:, None]) & (hist_idx < st.history.shape[1])
        st.history.scatter_(1, torch.where(hist_keep, hist_idx, st.history.shape[1] - 1), out[:, :width])
        rows = torch.arange(batch, device=dev)
        if not getattr(drafter, "observes", True):
            st.last.copy_(out[rows, n_acc.long()])
            st.kv_len.add_(torch.where(active, n_acc + 1, 0).to(st.kv_len.dtype))  # finished rows stay
            st.n_out.add_(n_acc + 1)
            return
        # ---- observe: drafter state for the committed columns + next root step ----
        path_w = path[:, :width].long()
        aux_path = {k: v.gather(1, path_w[..., None].expand(batch, width, v.shape[-1])) for k, v in aux.items()}
        fused = drafter.fuse(aux_path)  # [B, D+1, d]
        obs_tokens = torch.cat([st.last[:, None], out[:, :width]], 1)  # [B, D+2]
        sources = torch.cat([st.carry[:, None].to(fused.dtype), fused], 1)
        n_valid = (n_acc + 2).to(torch.int32)
        with phase("draft"):
            root_logits, root_state = drafter.observe(obs_tokens, sources, st.kv_len, n_valid, n_valid - 1)
        st.carry.copy_(fused[rows, n_acc.long()])
        st.last.copy_(out[rows, n_acc.long()])
        st.kv_len.add_(torch.where(active, n_acc + 1, 0).to(st.kv_len.dtype))  # finished rows stay
        st.n_out.add_(n_acc + 1)
        if root_logits is not None:
            st.root_logits.copy_(root_logits)
            st.root_state.copy_(root_state)

    # ---- drafting ----------------------------------------------------------------------------------------------
    def _draft_step_choice(self, logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor | None, torch.Tensor]:
        """A chain draft from draft-vocabulary logits ``[B, V_d]``: the target id, the draft distribution over the
        target vocabulary (rejection sampling only) and the drafter's top probability."""
        drafter = self.drafter
        if self.rejection:
            q = self.selector.probs(logits)
            u = torch.rand(q.shape[0], device=q.device)
            d = ops.sample(q.contiguous(), u)
            tok = drafter.to_target(d)
            ids = drafter.to_target(torch.arange(q.shape[-1], device=q.device))
            q_full = torch.zeros(q.shape[0], self.model.config.vocab_size, device=q.device)
            q_full[:, ids] = q
            return tok, q_full, q.gather(1, d[:, None])[:, 0]
        d = ops.argmax(logits)
        if not self.min_confidence:
            top = logits[:, 0]
        elif getattr(drafter, "confidence_measure", "top") == "gap":  # FREE: top-1 minus top-2 probability
            best = torch.softmax(logits.float(), -1).topk(2, -1).values
            top = best[:, 0] - best[:, 1]
        else:
            top = torch.softmax(logits.float(), -1).gather(1, d[:, None])[:, 0]
        return drafter.to_target(d), None, top

    def _draft_chain(self, st: _State) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]:
        drafter = self.drafter
        batch, dev = st.batch, st.kv_len.device
        k = self.depth
        tok, q, conf = self._draft_step_choice(st.root_logits)
        tokens, qs, confs = [tok], [q], [conf]
        state = st.root_state[:, None]
        base = st.kv_len + 1
        for d in range(1, k):
            bits = torch.full((batch, 1), (1 << d) - 1, dtype=torch.int64, device=dev)
            pos = (st.kv_len + d).to(torch.int32)[:, None]
            logits, out = drafter.tree_step(tok[:, None], state, pos, base, d, d - 1, bits)
            tok, q, conf = self._draft_step_choice(logits[:, 0])
            state = out
            tokens.append(tok)
            qs.append(q)
            confs.append(conf)
        drafts = torch.stack(tokens, 1)
        if self.min_confidence is not None:
            # stop after the first draft whose confidence is below the threshold (the first draft always stays)
            low = torch.stack(confs, 1) < self.min_confidence
            if getattr(drafter, "stop_inclusive", False):  # the low-confidence token itself goes to the exact pass
                stop = torch.cumsum(low.int(), 1) > 0
            else:
                stop = torch.cumsum(low.int(), 1) - low.int() > 0  # a low-confidence draft before this one
                stop[:, 0] = False
            drafts = torch.where(stop, torch.full_like(drafts, -1), drafts)
        parents = (torch.arange(k, device=dev) - 1).expand(batch, k).contiguous()  # -1: child of the root
        q_full = torch.stack(qs, 1) if self.rejection else None
        return drafts, parents, q_full

    # ---- verification ------------------------------------------------------------------------------------------
    def _choose(self, logits: torch.Tensor) -> torch.Tensor:
        """The exact model's token after every row of ``logits [..., V]``: argmax, or a draw from the selector."""
        if self.selector is None:
            return ops.argmax(logits)
        probs = self.selector.probs(logits)
        u = torch.rand(probs.shape[:-1], device=probs.device)
        return ops.sample(probs.contiguous(), u)

    def _pred(self, hidden: torch.Tensor) -> torch.Tensor:
        """The exact token after every row of final hidden states: greedy through the model's (possibly
        vocabulary-parallel) argmax, or a draw from the selector over the full logits."""
        if self.selector is None:
            return self.model.greedy(hidden)
        return self._choose(self.model.logits(hidden))

    def _verify(self, tokens: torch.Tensor, parents: torch.Tensor, hidden: torch.Tensor, drafts: torch.Tensor,
                q_full: torch.Tensor | None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        batch, length = tokens.shape
        dev = tokens.device
        plain_greedy = self.selector is None and not isinstance(self.verifier, TypicalVerifier)
        logits = None if plain_greedy else self.model.logits(hidden)  # [B, T, V]
        if self.rejection:
            p = self.selector.probs(logits).contiguous()  # [B, k + 1, V]
            k = drafts.shape[1]
            n_acc, out = ops.rejection(p, q_full.contiguous(), drafts.clamp_min(0),
                                       torch.rand(batch, k, device=dev), torch.rand(batch, device=dev))
            if self.min_confidence is not None or hasattr(self.drafter, "overlay"):  # invalid drafts never kept
                limit = (drafts >= 0).int().cumprod(1).sum(1).to(torch.int32)
                n_acc = torch.minimum(n_acc, limit)
            path = torch.arange(length, device=dev, dtype=torch.int32).expand(batch, length)
            path = torch.minimum(path, n_acc[:, None]).contiguous()
            return n_acc, path, out
        pred = self.model.greedy(hidden) if plain_greedy else self._choose(logits)  # [B, T]
        self.last_pred = pred  # read by drafters that learn from the target's predictions (lookahead's window)
        if self.accept_all:
            pred = torch.cat([drafts.clamp_min(0), pred[:, -1:]], 1)
            return ops.greedy_accept(tokens, parents, pred)
        if isinstance(self.verifier, TypicalVerifier):
            probs = torch.softmax(logits.float(), -1)
            parent_probs = probs.gather(1, parents[..., None].expand(batch, length, probs.shape[-1]))
            ok = self.verifier.acceptable(parent_probs, tokens) & (tokens >= 0)
            return ops.greedy_accept(tokens, parents, pred, ok)
        return ops.greedy_accept(tokens, parents, pred)

    def _draft_tree(self, st: _State) -> tuple[torch.Tensor, torch.Tensor]:
        drafter, tree = self.drafter, self.tree
        batch, dev = st.batch, st.kv_len.device
        k, depth = tree.topk, tree.depth
        # fused log-softmax + top-k (+ draft-to-target id map) per expansion: one kernel per step
        d2t = getattr(drafter, "d2t_map", None)

        def expand(logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
            vals, ids = ops.topk_logp(logits, k, LOGP_FLOOR, d2t)
            return vals, (ids if d2t is not None else drafter.to_target(ids))

        if dev.type == "cuda":
            return self._draft_tree_fused(st, expand)
        f_scores, f_tokens = expand(st.root_logits)  # frontier tokens [B, k]
        f_cand = torch.arange(k, device=dev).expand(batch, k)
        cand_tokens, cand_scores = [f_tokens], [f_scores]
        cand_parents = [torch.full((batch, k), -1, dtype=torch.int64, device=dev)]
        cand_depth = [torch.zeros(k, device=dev)]
        states = st.root_state[:, None].expand(batch, k, st.root_state.shape[-1]).contiguous()
        parent_fwd = torch.full((batch, k), -1, dtype=torch.int64, device=dev)
        fwd_bits = torch.zeros(batch, max(tree.forwarded, 1), dtype=torch.int64, device=dev)
        base = st.kv_len + 1
        for d in range(1, depth):
            f_idx = (d - 1) * k + torch.arange(k, device=dev)
            own = torch.ones(batch, k, dtype=torch.int64, device=dev) << f_idx[None]
            inherited = torch.where(parent_fwd >= 0, fwd_bits.gather(1, parent_fwd.clamp_min(0)),
                                    torch.zeros_like(own))
            bits = own | inherited
            fwd_bits[:, (d - 1) * k: d * k] = bits
            pos = (st.kv_len + d).to(torch.int32)[:, None].expand(batch, k).contiguous()
            logits, outs = drafter.tree_step(f_tokens, states, pos, base, d * k, (d - 1) * k, bits)
            c_vals, c_ids = expand(logits)
            child_scores = (f_scores[:, :, None] + c_vals).reshape(batch, k * k)
            child_tokens = c_ids.reshape(batch, k * k)
            child_parents = f_cand[:, :, None].expand(batch, k, k).reshape(batch, k * k)
            cand_tokens.append(child_tokens)
            cand_scores.append(child_scores)
            cand_parents.append(child_parents)
            cand_depth.append(torch.full((k * k,), float(d), device=dev))
            if d < depth - 1:
                pick = child_scores.topk(k, -1).indices
                origin = pick // k
                f_tokens = child_tokens.gather(1, pick)
                f_scores = child_scores.gather(1, pick)
                f_cand = k + (d - 1) * k * k + pick
                parent_fwd = (d - 1) * k + origin
                states = outs.gather(1, origin[..., None].expand(batch, k, outs.shape[-1]))
        tokens = torch.cat(cand_tokens, 1)
        scores = torch.cat(cand_scores, 1)
        parents = torch.cat(cand_parents, 1)
        depth_of = torch.cat(cand_depth)
        return select_candidates(tokens, scores, parents, depth_of, tree.total_tokens)

    def _draft_tree_fused(self, st: _State, expand) -> tuple[torch.Tensor, torch.Tensor]:
        """:meth:`_draft_tree` with the per-depth bookkeeping and the final selection in two CUDA kernels
        (``csrc/tree.cu``): the same candidates, frontiers, ancestor bits and tree, far fewer launches."""
        from ..ops._ext import require

        C = require()
        drafter, tree = self.drafter, self.tree
        batch, dev = st.batch, st.kv_len.device
        k, depth = tree.topk, tree.depth
        n_cand = k + (depth - 1) * k * k
        cand_tokens = torch.empty(batch, n_cand, dtype=torch.int64, device=dev)
        cand_scores = torch.empty(batch, n_cand, dtype=torch.float32, device=dev)
        cand_parents = torch.empty(batch, n_cand, dtype=torch.int64, device=dev)
        f_scores, f_tokens = expand(st.root_logits)
        f_scores = f_scores.contiguous()
        f_tokens = f_tokens.contiguous()
        cand_tokens[:, :k] = f_tokens
        cand_scores[:, :k] = f_scores
        cand_parents[:, :k] = -1
        f_cand = torch.arange(k, device=dev).expand(batch, k).contiguous()
        parent_fwd = torch.full((batch, k), -1, dtype=torch.int64, device=dev)
        fwd_bits = torch.zeros(batch, max(tree.forwarded, 1), dtype=torch.int64, device=dev)
        origin = torch.zeros(batch, k, dtype=torch.int64, device=dev)
        bits = (torch.ones(batch, k, dtype=torch.int64, device=dev) << torch.arange(k, device=dev)[None]).contiguous()
        fwd_bits[:, :k] = bits
        states = st.root_state[:, None].expand(batch, k, st.root_state.shape[-1]).contiguous()
        base = st.kv_len + 1
        for d in range(1, depth):
            pos = (st.kv_len + d).to(torch.int32)[:, None].expand(batch, k).contiguous()
            logits, outs = drafter.tree_step(f_tokens, states, pos, base, d * k, (d - 1) * k, bits)
            c_vals, c_ids = expand(logits)
            nxt = d < depth - 1
            new_bits = torch.empty_like(bits)
            C.tree_expand(c_vals.contiguous(), c_ids.contiguous(), f_scores, f_cand, f_tokens, parent_fwd, fwd_bits,
                          origin, new_bits, cand_tokens, cand_scores, cand_parents, d, nxt)
            if nxt:
                bits = new_bits
                states = outs.gather(1, origin[..., None].expand(batch, k, outs.shape[-1]))
        return C.tree_select(cand_tokens, cand_scores, cand_parents, k, tree.total_tokens)

    # ---- Sequoia static trees and SpecExec search -------------------------------------------------------------
    def _plan(self, device: torch.device) -> StaticPlan:
        plan = self._plans.get(device)
        if plan is None:  # built by the eager warm-up cycles, before any graph capture
            plan = self._plans[device] = StaticPlan(self.static_tree, device)
        return plan

    def _topk_ids(self, logits: torch.Tensor, k: int) -> torch.Tensor:
        """Target ids of the ``k`` most likely draft tokens of every row of ``logits [..., V_d]``."""
        d2t = getattr(self.drafter, "d2t_map", None)
        if k <= 16:
            _, ids = ops.topk_logp(logits, k, LOGP_FLOOR, d2t)
            return ids if d2t is not None else self.drafter.to_target(ids)
        return self.drafter.to_target(logits.topk(k, -1).indices)

    def _draft_static_tree(self, st: _State) -> tuple[torch.Tensor, torch.Tensor]:
        """Fill the Sequoia tree: every node is its parent's ``rank``-th most likely token; one draft step per depth
        over the nodes of that depth with children (economize ``decoding/sequoia.py:SequoiaDrafter.propose``)."""
        drafter, plan = self.drafter, self._plan(st.kv_len.device)
        batch = st.batch
        level = self._topk_ids(st.root_logits, plan.k[0])[:, plan.pick[0]]
        levels = [level]
        outs = None
        base = st.kv_len + 1
        for L in range(1, plan.depth):
            width, offset = plan.widths[L - 1], plan.offset[L - 1]
            tok = level[:, plan.fwd[L - 1]].contiguous()
            if L == 1:
                states = st.root_state[:, None].expand(batch, width, st.root_state.shape[-1]).contiguous()
            else:
                states = outs[:, plan.fwd_parent[L - 1]].contiguous()
            pos = (st.kv_len + L).to(torch.int32)[:, None].expand(batch, width).contiguous()
            bits = plan.bits[L - 1].expand(batch, width).contiguous()
            logits, outs = drafter.tree_step(tok, states, pos, base, offset + width, offset, bits)
            level = self._topk_ids(logits, plan.k[L]).reshape(batch, -1)[:, plan.pick[L]]
            levels.append(level)
        return torch.cat(levels, 1), plan.parents.expand(batch, plan.size)

    def _draft_search(self, st: _State) -> tuple[torch.Tensor, torch.Tensor]:
        """SpecExec: ``depth - 1`` best-first expansions of the ``width`` best open candidates, then the
        ``total_tokens`` best candidates (economize ``decoding/specexec.py:SpecExecDrafter``)."""
        drafter, opt = self.drafter, self.search
        batch, dev = st.batch, st.kv_len.device
        k, w = opt.topk, opt.width
        log_decay = math.log(opt.decay)
        d2t = getattr(drafter, "d2t_map", None)

        def expand(logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
            vals, ids = ops.topk_logp(logits, k, LOGP_FLOOR, d2t)
            return vals, (ids if d2t is not None else drafter.to_target(ids))

        n = opt.candidates
        tokens = torch.empty(batch, n, dtype=torch.int64, device=dev)
        scores = torch.empty(batch, n, dtype=torch.float32, device=dev)
        parents = torch.empty(batch, n, dtype=torch.int64, device=dev)
        depth = torch.empty(batch, n, dtype=torch.int64, device=dev)
        slot_of = torch.empty(batch, n, dtype=torch.int64, device=dev)  # forwarded slot of a candidate, -1: open
        vals, ids = expand(st.root_logits)
        tokens[:, :k] = ids
        scores[:, :k] = vals + log_decay
        parents[:, :k] = -1
        depth[:, :k] = 1
        slot_of[:, :k] = -1
        states = torch.empty(batch, 1 + opt.forwarded, st.root_state.shape[-1], dtype=st.root_state.dtype,
                             device=dev)
        states[:, 0] = st.root_state
        fwd_bits = torch.zeros(batch, opt.forwarded, dtype=torch.int64, device=dev)
        rows = torch.arange(batch, device=dev)[:, None]
        lanes = torch.arange(w, device=dev)
        base = st.kv_len + 1
        filled = k
        for s in range(opt.steps):
            pick = torch.where(slot_of[:, :filled] >= 0, float("-inf"), scores[:, :filled]).topk(w, -1).indices
            slot = s * w + lanes
            par = parents.gather(1, pick)
            par_slot = torch.where(par >= 0, slot_of.gather(1, par.clamp_min(0)), -1)
            inherited = torch.where(par_slot >= 0, fwd_bits.gather(1, par_slot.clamp_min(0)), 0)
            bits = (torch.ones(w, dtype=torch.int64, device=dev) << slot)[None] | inherited
            fwd_bits[:, s * w:(s + 1) * w] = bits
            slot_of.scatter_(1, pick, slot.expand(batch, w))
            node_depth = depth.gather(1, pick)
            pos = (st.kv_len[:, None] + node_depth).to(torch.int32)
            logits, outs = drafter.tree_step(tokens.gather(1, pick), states[rows, par_slot + 1].contiguous(), pos,
                                             base, (s + 1) * w, s * w, bits)
            states[:, 1 + s * w:1 + (s + 1) * w] = outs
            c_vals, c_ids = expand(logits)
            lo, hi = filled, filled + w * k
            tokens[:, lo:hi] = c_ids.reshape(batch, w * k)
            scores[:, lo:hi] = (scores.gather(1, pick)[:, :, None] + c_vals + log_decay).reshape(batch, w * k)
            parents[:, lo:hi] = pick[:, :, None].expand(batch, w, k).reshape(batch, w * k)
            depth[:, lo:hi] = (node_depth + 1)[:, :, None].expand(batch, w, k).reshape(batch, w * k)
            slot_of[:, lo:hi] = -1
            filled = hi
        return select_candidates(tokens, scores, parents, depth, opt.total_tokens)
