"""The block Walsh-Hadamard kernel (QuaRot's online rotation) and its fusion into the gated activation, against the
fp32 PyTorch transform; a rotated model on the GPU against the same model unrotated."""

import pytest
import torch

import economize_b200 as eco
from economize_b200 import ops
from economize_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _dense_h(block: int, device) -> torch.Tensor:
    h = torch.ones(1, 1, dtype=torch.float64)
    while h.shape[0] < block:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return (h / block ** 0.5).float().to(device)


@pytest.mark.parametrize("rows,F,block", [(1, 14336, 2048), (61, 14336, 2048), (5, 688, 16), (3, 4096, 4096),
                                          (2, 8192, 8192), (7, 96, 32), (4, 11008, 256)])
def test_hadamard_matches_fp32(cuda, rows, F, block):
    g = torch.Generator(device=cuda).manual_seed(rows + F)
    x = torch.randn(rows, F, device=cuda, generator=g).bfloat16()
    y = ops.hadamard(x, block)
    want = (x.float().view(rows, F // block, block) @ _dense_h(block, cuda)).view(rows, F)
    torch.testing.assert_close(y.float(), want, atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(y.float(), ref.hadamard(x.float(), block), atol=2e-2, rtol=1e-2)
    # an orthogonal, symmetric transform: applying it twice gives x back up to the two roundings
    torch.testing.assert_close(ops.hadamard(y, block).float(), x.float(), atol=3e-2, rtol=2e-2)


@pytest.mark.parametrize("act", ["silu", "gelu_tanh", "clamped_swiglu"])
def test_glu_hadamard_equals_glu_then_hadamard(cuda, act):
    g = torch.Generator(device=cuda).manual_seed(2)
    gu = torch.randn(61, 2 * 14336, device=cuda, generator=g).bfloat16()
    fused = ops.glu(gu, act, 7.0, hadamard=2048)
    assert torch.equal(fused, ops.hadamard(ops.glu(gu, act, 7.0), 2048))
    want = ref.hadamard(ref.glu(gu.float(), act, 7.0), 2048)
    torch.testing.assert_close(fused.float(), want, atol=3e-2, rtol=2e-2)


def test_glu_hadamard_reduces_split_k_partials(cuda):
    g = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(61, 4096, device=cuda, generator=g).bfloat16()
    w = (torch.randn(2 * 2048, 4096, device=cuda, generator=g) * 0.02).bfloat16()
    p = ops.linear_parts(x, w)
    assert isinstance(p, ops.Partials)
    assert torch.equal(ops.glu(p, "silu", hadamard=512), ops.glu(p.sum(), "silu", hadamard=512))


def test_bad_blocks_are_refused(cuda):
    x = torch.randn(2, 96, device=cuda).bfloat16()
    for block in (64, 12, 4, 16384):
        with pytest.raises(RuntimeError, match="power of two"):
            ops.require().hadamard(x if block != 16384 else torch.zeros(1, 16384, device=cuda).bfloat16(), block)


def test_rotated_model_keeps_its_function_on_gpu(cuda):
    from economize_b200.models.config import tiny_llama
    from economize_b200.models.llama import CausalLM, init_weights
    from economize_b200.techniques.rotate import RotateConfig

    cfg = tiny_llama(hidden_size=512, num_heads=4, num_kv_heads=2, head_dim=128, intermediate_size=1536)
    ids = torch.randint(0, cfg.vocab_size, (1, 40), device=cuda, generator=torch.Generator(device=cuda).manual_seed(0))
    base = eco.apply(init_weights(CausalLM(cfg, torch.bfloat16, cuda), seed=0))(ids).float()
    rot = eco.apply(init_weights(CausalLM(cfg, torch.bfloat16, cuda), seed=0), RotateConfig())
    assert rot.model.layers[0].down_hadamard == 512
    out = rot(ids).float()
    assert (out - base).norm() / base.norm() < 0.05
    assert (out.argmax(-1) == base.argmax(-1)).float().mean() > 0.9


def test_hadamard_of_a_misaligned_view(cuda):
    buf = torch.randn(3 * 64 + 1, device=cuda).bfloat16()
    x = buf[1:].view(3, 64)  # contiguous, 2 bytes past a 16-byte boundary
    assert x.data_ptr() % 16 != 0
    torch.testing.assert_close(ops.hadamard(x, 64).float(), ref.hadamard(x.float(), 64), atol=2e-2, rtol=1e-2)
    gu = torch.randn(2 * 2 * 64 + 1, device=cuda).bfloat16()[1:].view(2, 128)
    want = ref.hadamard(ref.glu(gu.float(), "silu"), 64)
    torch.testing.assert_close(ops.glu(gu, "silu", hadamard=64).float(), want, atol=3e-2, rtol=2e-2)
