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


def _naive_vs_keep(cols, offsets, base, t, limit, size):
    keep = torch.zeros(*cols.shape[:-1], size, dtype=torch.bool)
    j = torch.arange(size)
    for idx in torch.cartesian_prod(*[torch.arange(n) for n in cols.shape[:-1]]).reshape(-1, cols.dim() - 1):
        idx = tuple(idx.tolist())
        row = torch.zeros(size, dtype=torch.bool)
        for c in cols[idx].tolist():
            if 0 <= c < size:
                row[c] = True
        for o in offsets[idx].tolist():
            row |= (j >= base - o) & (j < base + t - o)
        keep[idx] = row & (j < limit)
    return keep


def _bits(words, size):
    return ((words.long()[..., None] >> torch.arange(32)) & 1).bool().reshape(*words.shape[:-1], size)


def test_vs_keep_reference_matches_the_definition():
    from economize_b200.ops import reference

    g = torch.Generator().manual_seed(0)
    size, base, t = 512, 300, 64
    cols = torch.randint(-3, size + 5, (2, 3, 40), generator=g)
    offsets = torch.randint(-10, 400, (2, 3, 25), generator=g)
    for limit in (base, 129, 0):
        got = _bits(reference.vs_keep(cols, offsets, base, t, limit, size), size)
        assert torch.equal(got, _naive_vs_keep(cols, offsets, base, t, limit, size))


@pytest.mark.gpu
@pytest.mark.parametrize("size,nv,ns", [(512, 40, 25), (131072, 1000, 1000), (4096, 0, 64), (2048, 30, 0)])
def test_vs_keep_kernel_matches_reference(cuda, size, nv, ns):
    from economize_b200 import ops
    from economize_b200.ops import reference

    g = torch.Generator().manual_seed(size + nv)
    base, t = size - size // 4, min(2048, size // 4)
    cols = torch.randint(-3, size + 5, (2, 8, nv), generator=g)
    offsets = torch.randint(-10, size, (2, 8, ns), generator=g)
    for limit in (base, base - 7):
        got = ops.vs_keep(cols.to(cuda), offsets.to(cuda), base, t, limit, size)
        assert torch.equal(got.cpu(), reference.vs_keep(cols, offsets, base, t, limit, size))
