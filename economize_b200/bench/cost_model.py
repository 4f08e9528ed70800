"""Analytic cost model of a decode step: FLOPs and bytes per pass, and the roofline time on a hardware preset
(economize ``bench/cost_model.py:110-600``; its presets stop at the H100, this one adds the B200 with the peaks
measured on the benchmark pool).

Memory-bound decode reads every weight once per pass plus the KV cache of every row; compute is ``2 * params``
FLOPs per token plus attention. The roofline time of a pass is ``max(bytes / HBM bandwidth, flops / tensor peak)``;
for tensor parallelism the per-rank weights shrink by the TP degree and every row-parallel projection adds an
all-reduce of ``[tokens, hidden]`` bf16 over NVLink.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

__all__ = ["HARDWARE", "Hardware", "decode_step_cost", "load_measured", "roofline"]


@dataclass(frozen=True)
class Hardware:
    name: str
    hbm_gbs: float          # achievable copy bandwidth (GB/s)
    bf16_tflops: float      # dense bf16 tensor throughput (TFLOP/s)
    link_gbs: float = 0.0   # per-direction GPU-to-GPU bandwidth (GB/s)
    hbm_gb: float = 0.0


HARDWARE: dict[str, Hardware] = {
    "a100-40gb": Hardware("a100-40gb", 1400.0, 312.0, 300.0, 40.0),
    "a100-80gb": Hardware("a100-80gb", 1800.0, 312.0, 300.0, 80.0),
    "h100-sxm": Hardware("h100-sxm", 3000.0, 989.0, 450.0, 80.0),
    # B200: measured copy bandwidth and cuBLAS bf16 (burst) on the pool, peer copy 770 GB/s per direction
    "b200": Hardware("b200", 6539.2, 1657.8, 770.0, 180.0),
}


def load_measured(path: str | Path) -> Hardware:
    """A preset from a measured-peaks JSON file (``hbm_gbs``, ``bf16_tflops``)."""
    data = json.loads(Path(path).read_text())
    return Hardware(data.get("gpu_name", "measured"), float(data["hbm_gbs"]), float(data["bf16_tflops"]), 770.0,
                    180.0)


def decode_step_cost(config, tokens: int, kv_tokens: int, tp: int = 1, weight_bits: int = 16,
                     kv_bits: int = 16) -> dict[str, float]:
    """FLOPs, HBM bytes and NVLink bytes per rank of one pass over ``tokens`` new tokens attending to
    ``kv_tokens`` cached tokens in total (summed over rows)."""
    h, f, layers = config.hidden_size, config.intermediate_size, config.num_layers
    qkv = h * (config.q_size + 2 * config.kv_size)
    proj = qkv + config.q_size * h + 3 * h * f
    head = config.vocab_size * h
    weights = layers * proj / tp + head / tp
    flops = 2 * tokens * weights + layers * 4 * tokens * kv_tokens * config.head_dim * config.num_heads / tp
    weight_bytes = weights * weight_bits / 8
    kv_bytes = layers * 2 * kv_tokens * config.kv_size / tp * kv_bits / 8
    act_bytes = layers * tokens * h * 2 * 6
    link = 0.0 if tp == 1 else layers * 2 * tokens * h * 2 * (tp - 1) / tp * 2
    return {"flops": flops, "hbm_bytes": weight_bytes + kv_bytes + act_bytes, "link_bytes": link}


def roofline(cost: dict[str, float], hw: Hardware) -> dict[str, float]:
    """Lower-bound time (seconds) of each resource and the bound."""
    t_mem = cost["hbm_bytes"] / (hw.hbm_gbs * 1e9)
    t_math = cost["flops"] / (hw.bf16_tflops * 1e12)
    t_link = cost.get("link_bytes", 0.0) / (hw.link_gbs * 1e9) if hw.link_gbs else 0.0
    return {"memory_s": t_mem, "compute_s": t_math, "link_s": t_link, "bound_s": max(t_mem, t_math, t_link)}
