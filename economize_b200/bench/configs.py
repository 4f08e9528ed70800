"""The benchmark configurations of the B200 build's north star, composed from the public API.

Each builder returns a :class:`BenchSpec`: the accelerated model (``apply`` of the configuration's techniques to a
random-init target of the named architecture), its decoding configuration, the synthetic prompts and the number of
new tokens. ``scale="tiny"`` keeps every technique and the composition but shrinks the architecture, so the same
code runs on the CPU in tests; ``scale="full"`` is the named architecture.

1. CPU fp32 plumbing: the 4-layer Llama-style target + EAGLE-3, a greedy chain of 4 drafts, prompts of 17 and 40
   tokens, 32 new tokens; the output must equal plain greedy decoding.
2. Llama-3.1-8B + EAGLE-3 dynamic tree (depth 6, 60 nodes): ``bench.py``'s default path (both arms).
3. Llama-3.1-70B architecture with ShortGPT removing 8 blocks, int4 group-128 weights in the GPTQ layout, fp8 e4m3
   KV with per-head scales, and an EAGLE-3 drafter with int8 weights (tensor parallel over the ranks given).
4. Mixtral-8x7B-style MoE (8 experts, top-2) with block-scaled fp8 attention projections (128 x 128 weight / 1 x 128
   activation scales) + 4 Medusa heads, experts over the expert-parallel group when one is given.
5. Long context: Llama-3.1-8B target with 2-bit KIVI KV, a 1B-scale draft LM (16 layers, hidden 2048) on another
   device whose own cache is a StreamingLLM view (sink + recent window), drafts handed over by peer copies.

The reference states these recipes as composed techniques (``/root/reference/README.md:70-84``,
``techniques/sparse_kv_draft``, ``techniques/placed_draft/drafter.py:23-80``); the reference publishes no number for
configurations 3-5.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch

__all__ = ["BenchSpec", "CONFIGS", "build", "config1", "config3", "config4", "config5"]


@dataclass
class BenchSpec:
    name: str
    model: Any  # EfficientModel
    decoding: Any  # DecodeConfig
    prompts: list[torch.Tensor]
    new_tokens: int
    notes: dict[str, Any] = field(default_factory=dict)

    def step(self):
        """One benchmark step: generate ``new_tokens`` after every prompt through the public API."""
        return self.model.decode_batch(self.prompts, self.new_tokens, decoding=self.decoding)


def _prompts(batch: int, length: int, vocab: int, device, seed: int = 1234) -> list[torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (length,), generator=g).to(device) for _ in range(batch)]


def _target(cfg, dtype, device, seed: int = 0, tp=None):
    from ..models.llama import CausalLM, init_weights

    model = init_weights(CausalLM(cfg, dtype, device), seed=seed, scaled_residual=True)
    if tp is not None and tp.size > 1:
        from ..distributed import tensor_parallel

        tensor_parallel(model, tp, fused=device != "cpu" and torch.device(device).type == "cuda")
    return model


def config1(device: str | torch.device = "cpu") -> BenchSpec:
    """The CPU fp32 plumbing configuration (scale is fixed by its definition)."""
    import economize_b200 as eco
    from ..models.config import tiny_llama
    from ..models.llama import CausalLM, init_weights
    from ..techniques.eagle3 import Eagle3Config

    cfg = tiny_llama(hidden_size=256, num_heads=4, num_kv_heads=2, intermediate_size=688, vocab_size=1024,
                     num_layers=4, rope_theta=1e4)
    dtype = torch.float32 if torch.device(device).type == "cpu" else torch.bfloat16
    model = init_weights(CausalLM(cfg, dtype, device), seed=0, std=0.02)
    em = eco.apply(model, Eagle3Config())
    prompts = [torch.randint(0, 1024, (n,), generator=torch.Generator().manual_seed(n)).to(device) for n in (17, 40)]
    return BenchSpec("1: CPU fp32 plumbing (4-layer Llama-style + EAGLE-3, chain of 4)", em,
                     eco.DecodeConfig(cycle_length=5), prompts, 32,
                     {"check": "tokens equal plain greedy decoding"})


def config3(scale: str = "full", device: str | torch.device = "cuda", tp=None, batch: int = 16,
            prompt_len: int = 2048, new_tokens: int = 512, calibration_rows: int = 4) -> BenchSpec:
    """70B architecture, ShortGPT(8 blocks), int4 g128 (GPTQ layout), fp8 per-head KV, int8 EAGLE-3 drafter.

    Weights are random, so the int4 grid is fitted by round to nearest (GPTQ's Hessian correction changes values,
    not the stored format or the kernel that reads it); under tensor parallelism every rank quantizes its own shard
    (round to nearest of a 128-column group is the same before and after sharding along either dimension)."""
    import economize_b200 as eco
    from ..models.config import llama31_70b, tiny_llama
    from ..techniques.eagle3 import Eagle3Config
    from ..techniques.kv_quant import KVFp8Config
    from ..techniques.prune.config import DepthPruneConfig
    from ..techniques.quant.config import DraftQuantConfig, QuantConfig

    if scale == "full":
        cfg, removed = llama31_70b(), 8
    else:
        # head dimension 128: the fp8 cache kernels' width
        cfg = tiny_llama(hidden_size=256, num_heads=2, num_kv_heads=1, head_dim=128, intermediate_size=512,
                         num_layers=10, vocab_size=1024)
        removed = 2
    dtype = torch.bfloat16 if torch.device(device).type == "cuda" else torch.float32
    model = _target(cfg, dtype, device)
    calib = torch.stack(_prompts(calibration_rows, min(prompt_len, 256), cfg.vocab_size, device, seed=99))
    prune = DepthPruneConfig(method="shortgpt", num_blocks=removed)
    rest = (QuantConfig(format="int4", method="rtn", group_size=128), KVFp8Config(format="e4m3", scale="head"),
            Eagle3Config(), DraftQuantConfig(format="int8"))
    if tp is None or tp.size == 1:
        em = eco.apply(model, prune, *rest, calibration=calib)
        chosen = em.techniques["depth_prune"].config.layers
    else:
        # depth pruning measures block influence on the whole (unsharded) model; then the shards are cut and every
        # rank quantizes its own
        from ..distributed import tensor_parallel

        pruned = eco.apply(model, prune, calibration=calib)
        chosen = pruned.techniques["depth_prune"].config.layers
        tensor_parallel(pruned.model, tp, fused=torch.device(device).type == "cuda")
        em = eco.apply(pruned.model, *rest, calibration=calib)
    decoding = eco.DecodeConfig(cycle_length=7, draft_policy="dynamic_tree",
                                draft_policy_options={"depth": 6, "topk": 10, "total_tokens": 60})
    return BenchSpec("3: Llama-3.1-70B arch, ShortGPT -8, int4 g128, fp8 KV, int8 EAGLE-3", em, decoding,
                     _prompts(batch, prompt_len, cfg.vocab_size, device), new_tokens,
                     {"removed_blocks": list(chosen), "quant": "int4 g128 (GPTQ layout, round to nearest)",
                      "kv": "fp8 e4m3, per-head scales", "drafter": "EAGLE-3, int8 weights",
                      "tp": 1 if tp is None else tp.size})


def config4(scale: str = "full", device: str | torch.device = "cuda", ep=None, batch: int = 64,
            prompt_len: int = 1024, new_tokens: int = 256) -> BenchSpec:
    """Mixtral-8x7B-style MoE, block-scaled fp8 attention projections, 4 Medusa heads, expert parallelism."""
    import economize_b200 as eco
    from ..models.config import mixtral_8x7b, tiny_llama
    from ..techniques.medusa import MedusaConfig
    from ..techniques.quant.config import QuantConfig

    if scale == "full":
        cfg = mixtral_8x7b()
    else:
        cfg = tiny_llama(hidden_size=256, num_heads=4, num_kv_heads=2, intermediate_size=256, num_layers=3,
                         vocab_size=1024, num_experts=8, experts_per_token=2, model_type="mixtral")
    dtype = torch.bfloat16 if torch.device(device).type == "cuda" else torch.float32
    model = _target(cfg, dtype, device)
    if ep is not None and ep.size > 1:
        # every rank keeps its block of experts and decodes its own share of the batch; the MoE layers dispatch
        # rows to the experts' owners and combine the results over the expert-parallel group
        own = ep.owned(cfg.num_experts)
        for layer in model.layers:
            layer.w_gate_up.data = layer.w_gate_up.data[own.start:own.stop].contiguous()
            layer.w_down.data = layer.w_down.data[own.start:own.stop].contiguous()
        if hasattr(ep, "setup"):
            ep.setup(cfg.hidden_size, len(own), cfg.experts_per_token)
        model.ep = ep
        batch = max(1, batch // ep.size)
    configs = [MedusaConfig(num_heads=4)]
    if torch.device(device).type == "cuda":  # the block-scaled fp8 GEMM is a tcgen05 kernel (no CPU path)
        configs.insert(0, QuantConfig(format="fp8_block", method="rtn"))
    em = eco.apply(model, *configs)
    decoding = eco.DecodeConfig(cycle_length=5, draft_policy="fixed", verifier="typical")
    return BenchSpec("4: Mixtral-8x7B-style MoE, block fp8 attention, Medusa-4", em, decoding,
                     _prompts(batch, prompt_len, cfg.vocab_size, device), new_tokens,
                     {"weights": "fp8 128x128 blocks (attention projections); experts bf16",
                      "drafter": "Medusa, 4 heads", "ep": None if ep is None else getattr(ep, "world", None)})


def config5(scale: str = "full", device: str | torch.device = "cuda", draft_device: str | torch.device | None = None,
            batch: int = 4, prompt_len: int = 131072, new_tokens: int = 256, window: int = 2048,
            sink: int = 16) -> BenchSpec:
    """128K context: KIVI 2-bit target KV, a 1B-scale draft LM on another device with a StreamingLLM cache view."""
    import economize_b200 as eco
    from ..models.config import llama31_8b, tiny_llama
    from ..models.llama import CausalLM, init_weights
    from ..techniques.kv_quant import KIVIConfig
    from ..techniques.placed_draft import PlacedDraftModelConfig

    if scale == "full":
        cfg = llama31_8b()
        dcfg = llama31_8b(num_layers=16, hidden_size=2048, num_heads=32, num_kv_heads=8, head_dim=64,
                          intermediate_size=8192)
    else:
        # head dimension 128: the KIVI kernels' width
        cfg = tiny_llama(num_layers=4, num_heads=2, num_kv_heads=1, head_dim=128, vocab_size=1024,
                         max_position_embeddings=8192)
        dcfg = tiny_llama(num_layers=2, hidden_size=128, num_heads=2, num_kv_heads=1, head_dim=64,
                          intermediate_size=256, vocab_size=1024, max_position_embeddings=8192)
    draft_device = draft_device or device
    dtype = torch.bfloat16 if torch.device(device).type == "cuda" else torch.float32
    target = _target(cfg, dtype, device)
    draft = init_weights(CausalLM(dcfg, dtype, draft_device), seed=5, scaled_residual=True)
    em = eco.apply(target, KIVIConfig(bits=2, residual=128),
                   PlacedDraftModelConfig(model=draft, device=str(draft_device), sink=sink, window=window))
    decoding = eco.DecodeConfig(cycle_length=6)
    return BenchSpec("5: 128K context, KIVI-2 target KV, placed 1B draft LM with a StreamingLLM cache", em,
                     decoding, _prompts(batch, prompt_len, cfg.vocab_size, device), new_tokens,
                     {"kv": "KIVI 2-bit, residual 128", "draft": f"{dcfg.num_layers} layers, hidden {dcfg.hidden_size}"
                      f", on {draft_device}, cache view sink {sink} + window {window}"})


CONFIGS = {1: config1, 3: config3, 4: config4, 5: config5}


def build(number: int, **kwargs) -> BenchSpec:
    if number not in CONFIGS:
        raise ValueError(f"configuration {number} is built by bench.py's default path" if number == 2 else
                         f"no benchmark configuration {number}")
    return CONFIGS[number](**kwargs)
