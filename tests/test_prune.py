"""Pruning: masks (magnitude / Wanda / SparseGPT, unstructured and N:M), 2:4 compressed storage and its kernel,
depth pruning (ShortGPT / SLEB) and their composition with drafters and checkpoints."""

import pytest
import torch

import economize_b200 as eco
from economize_b200.ops.sparse import Sparse24Weight, mask_24, pack_24, unpack_24
from economize_b200.techniques.eagle3 import Eagle3Config
from economize_b200.techniques.prune import DepthPruneConfig, PruneConfig, nm_mask, sparsegpt, unstructured_mask

from .helpers import prompts, reference_greedy, tiny_model

CAL = torch.randint(0, 1024, (2, 32), generator=torch.Generator().manual_seed(4))


def test_pack_24_roundtrip_with_sparse_groups():
    w = torch.randn(4, 128)
    m = mask_24(w.abs())
    m[0, :4] = torch.tensor([False, True, False, False])  # a group keeping one entry
    v, meta = pack_24(w, m)
    assert torch.equal(unpack_24(v, meta), w * m)


def test_masks():
    s = torch.rand(3, 16)
    assert (nm_mask(s, 2, 4).reshape(3, 4, 4).sum(-1) == 2).all()
    assert (unstructured_mask(s, 0.25).sum(-1) == 12).all()


def test_sparsegpt_beats_magnitude():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(1024, 128, generator=g) @ (torch.randn(128, 128, generator=g) / 11)
    w = torch.randn(64, 128, generator=g) * 0.02
    ref = x @ w.t()
    mag = w * nm_mask(w.abs(), 2, 4)
    sg, keep = sparsegpt(w, x.t() @ x, 0.5, (2, 4))
    assert (keep.reshape(64, -1, 4).sum(-1) == 2).all()
    assert (x @ sg.t() - ref).norm() < 0.85 * (x @ mag.t() - ref).norm()


@pytest.mark.parametrize("method", ["magnitude", "wanda", "sparsegpt"])
def test_prune_24_decodes_and_stores_compressed(method):
    model = tiny_model()
    eff = eco.apply(model, PruneConfig(method=method, sparsity="2:4"), calibration=CAL)
    assert isinstance(eff.model.layers[0].wqkv, Sparse24Weight)
    assert abs(eff.techniques["prune"].sparsity() - 0.5) < 0.02
    p = prompts((15,))[0]
    assert torch.equal(eff.decode(p, 8).tokens, reference_greedy(eff.model, p, 8))


def test_prune_unstructured_masks_in_place(tmp_path):
    model = tiny_model()
    eff = eco.apply(model, PruneConfig(method="magnitude", sparsity=0.3))
    w = eff.model.layers[1].wo
    assert isinstance(w, torch.nn.Parameter) and abs(float((w == 0).float().mean()) - 0.3) < 0.02
    eff.save_pretrained(str(tmp_path))
    loaded = eco.load(tiny_model(), str(tmp_path))
    assert set(loaded.techniques["prune"].masks) == set(eff.techniques["prune"].masks)


@pytest.mark.parametrize("method", ["shortgpt", "sleb"])
def test_depth_prune_then_drafter(method):
    model = tiny_model()
    eff = eco.apply(model, DepthPruneConfig(method=method, num_blocks=1), Eagle3Config(), calibration=CAL,
                    decoding=eco.DecodeConfig(cycle_length=4))
    assert eff.model.config.num_layers == 3 and len(eff.model.layers) == 3
    removed = eff.techniques["depth_prune"].removed
    assert len(removed) == 1 and 0 < removed[0] < 3
    assert max(eff.techniques["eagle3"].aux_layers) <= 3
    p = prompts((17,))[0]
    assert torch.equal(eff.decode(p, 8).tokens, reference_greedy(eff.model, p, 8))


def test_depth_prune_checkpoint_replays(tmp_path):
    eff = eco.apply(tiny_model(), DepthPruneConfig(num_blocks=2), calibration=CAL)
    eff.save_pretrained(str(tmp_path))
    loaded = eco.load(tiny_model(), str(tmp_path))
    assert loaded.techniques["depth_prune"].removed == eff.techniques["depth_prune"].removed
    assert loaded.model.config.num_layers == 2


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (61, 6144, 4096), (200, 512, 1024), (7, 264, 512)])
def test_linear_sp24_matches_dense(cuda, M, N, K):
    g = torch.Generator(device=cuda).manual_seed(0)
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.02).bfloat16()
    sw = Sparse24Weight.from_dense(w)
    x = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    y = sw.linear(x)
    exact = x.float() @ sw.dequantize(torch.float32).t()
    torch.testing.assert_close(y.float(), exact, atol=2e-2, rtol=2e-2)


def test_width_prune_recovery_lora_trains_and_reloads(tmp_path):
    """LLM-Pruner's recovery stage: an always-on LoRA of the pruned layers, trained with next-token cross-entropy,
    lowers the pruned model's loss on the training tokens and reloads from a checkpoint."""
    import economize_b200 as eco
    from economize_b200.techniques.width_prune import WidthPruneConfig
    from economize_b200.train import fit
    from economize_b200.train.objective import RecoveryCE

    from .helpers import tiny_model

    model = tiny_model()
    data = torch.randint(0, 1024, (8, 48), generator=torch.Generator().manual_seed(3))
    em = eco.apply(model, WidthPruneConfig(ratio=0.5, recovery_rank=8), calibration=data[:2])
    tech = em.techniques["width_prune"]
    assert len(tech.recovery) == 4 * model.config.num_layers and tech.lora_targets()
    before, _ = RecoveryCE(em).loss(data)
    fit(em, data, steps=40, batch_size=4, lr=3e-3, warmup_steps=2, log_every=100)
    after, _ = RecoveryCE(em).loss(data)
    assert float(after.detach()) < float(before.detach())
    out = em.decode_batch([data[0, :10]], 6, decoding=eco.DecodeConfig(cycle_length=1))[0]
    em.save_pretrained(tmp_path)
    em2 = eco.load(tiny_model(), tmp_path)
    out2 = em2.decode_batch([data[0, :10]], 6, decoding=eco.DecodeConfig(cycle_length=1))[0]
    assert torch.equal(out.tokens, out2.tokens)
