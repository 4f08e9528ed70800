"""MInference: patterns that keep every key reproduce the dense prefill, sparse patterns hide keys and change the
prefill only a little, and the attention kernel's chunk skipping matches the reference attention."""

import pytest
import torch

import economize_b200 as eco
from economize_b200.runtime.cache import StepBatch
from economize_b200.techniques.minference import MInferenceConfig

from .helpers import tiny_model


def _hidden(model, tokens):
    b, s = tokens.shape
    cache = model.new_cache(b, ((s + 127) // 128) * 128)
    lengths = torch.full((b,), s, dtype=torch.int32, device=tokens.device)
    h, _ = model.forward_step(tokens, StepBatch.prefill(lengths, s), cache)
    return h.float()


TOKENS = torch.randint(0, 1024, (2, 640), generator=torch.Generator().manual_seed(0))


@pytest.mark.parametrize("cfg", [MInferenceConfig(pattern="a_shape", sinks=0, local=4096, chunk=128),
                                 MInferenceConfig(pattern="block_sparse", top_k=100, chunk=256),
                                 MInferenceConfig(pattern="vertical_slash", vertical=4096, slash=4096, chunk=128)])
def test_full_patterns_equal_dense(cfg):
    dense = _hidden(tiny_model(), TOKENS)
    m = tiny_model()
    eco.apply(m, cfg)
    torch.testing.assert_close(_hidden(m, TOKENS), dense, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("cfg", [MInferenceConfig(pattern="a_shape", sinks=16, local=128, chunk=128),
                                 MInferenceConfig(pattern="block_sparse", top_k=2, chunk=128),
                                 MInferenceConfig(pattern="vertical_slash", vertical=30, slash=100, chunk=128)])
def test_sparse_patterns_approximate_dense(cfg):
    dense = _hidden(tiny_model(), TOKENS)
    m = tiny_model()
    em = eco.apply(m, cfg)
    out = _hidden(m, TOKENS)
    rel = (out - dense).norm() / dense.norm()
    assert 0 < rel < 0.5, float(rel)
    assert em.decode(TOKENS[0, :300], 4).tokens.numel() == 4  # decoding after a sparse prefill


@pytest.mark.gpu
def test_sparse_prefill_on_gpu_matches_reference_attention(cuda):
    """The kernel's skipping of hidden key chunks gives the masked attention of the CPU reference (same weights)."""
    from economize_b200.models.llama import CausalLM

    from .helpers import gpu_tiny_model

    tokens = torch.randint(0, 1024, (1, 1024), generator=torch.Generator().manual_seed(1)).to(cuda)
    m = gpu_tiny_model(cuda)
    cpu = CausalLM(m.config, torch.float32, "cpu")
    cpu.load_state_dict({k: v.float().cpu() for k, v in m.state_dict().items()})
    cfg = MInferenceConfig(pattern="a_shape", sinks=128, local=256, chunk=256)
    eco.apply(m, cfg)
    eco.apply(cpu, cfg)
    h = _hidden(m, tokens).cpu()
    h_ref = _hidden(cpu, tokens.cpu())
    rel = (h - h_ref).norm() / h_ref.norm()
    assert rel < 0.05, float(rel)
    dense = _hidden(gpu_tiny_model(cuda), tokens).cpu()
    assert (h - dense).norm() / dense.norm() > 2 * rel  # the pattern did hide keys
