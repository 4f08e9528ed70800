"""Activation sparsity: TEAL (thresholds, greedy allocation, phase policies), CATS and Deja Vu on the CPU with the
masked dense backend, and the CUDA kernels (colsparse_linear, glu_rows) against PyTorch fp32 references."""

import pytest
import torch
import torch.nn.functional as F

import economize_b200 as eco
from economize_b200.ops.act_sparse import (PhasePolicy, TealWeight, apply_mode, block_sparsity, greedy_allocation,
                                           magnitude_quantile, sparsify)
from economize_b200.runtime.phase import phase
from economize_b200.techniques.mlp_sparsity import CatsConfig, DejaVuConfig
from economize_b200.techniques.sparsity import TealConfig

from .helpers import prompts, tiny_model

CAL = torch.randint(0, 1024, (2, 48), generator=torch.Generator().manual_seed(3))


def test_policy_modes():
    p = PhasePolicy.coerce("second_half")
    assert p.mode("prefill", 9) == "second_half" and p.mode("decode", 1) == "all" and p.mode("draft", 4) == "all"
    assert p.mode(None, 1) == "all" and p.mode(None, 7) == "second_half"
    assert PhasePolicy.coerce({"decode": "dense"}).mode("decode", 1) == "dense"
    with pytest.raises(eco.ConfigError):
        PhasePolicy.coerce("half")


def test_sparsify_and_modes():
    x = torch.tensor([[[0.1, -0.5, 0.2], [0.3, 0.05, -0.7]]])
    assert torch.equal(sparsify(x, 0.2), torch.tensor([[[0.0, -0.5, 0.0], [0.3, 0.0, -0.7]]]))
    half = apply_mode(x, 0.2, "second_half")
    assert torch.equal(half[0, 0], x[0, 0]) and torch.equal(half[0, 1], sparsify(x, 0.2)[0, 1])


def test_quantile_and_greedy():
    mags = torch.arange(1, 101, dtype=torch.float32)
    assert magnitude_quantile(mags, 0.4) == 40.0 and magnitude_quantile(mags, 0.0) == 0.0
    sizes = {"a": 100, "b": 300}

    def err(levels):  # map b is cheap to sparsify
        return levels["a"] * 10 + levels["b"]

    levels, path = greedy_allocation(err, sizes, 0.5, step=0.1, unit=100)
    assert block_sparsity(levels, sizes) >= 0.5 - 1e-9
    assert levels["b"] > levels["a"] and all(s.name == "b" for s in path[:3])


@pytest.mark.parametrize("allocation", ["uniform", "greedy"])
def test_teal_reaches_target_and_detaches(allocation):
    model = tiny_model()
    before = {k: v.clone() for k, v in model.state_dict().items()}
    eff = eco.apply(model, TealConfig(sparsity=0.4, allocation=allocation, backend="dense", greedy_step=0.1),
                    calibration=CAL)
    tech = eff.techniques["teal"]
    assert tech.calibrated
    layer = model.layers[0]
    sizes = {m: getattr(layer, m).shape[0] * getattr(layer, m).shape[1] for m in ("wqkv", "wo", "w_gate_up",
                                                                                   "w_down")}
    lv = dict(zip(("wqkv", "wo", "w_gate_up", "w_down"), tech.levels[0].tolist()))
    assert block_sparsity(lv, sizes) == pytest.approx(0.4, abs=0.06)
    out = eff.decode(prompts((20,))[0], 6)
    assert out.tokens.numel() == 6
    assert isinstance(model.layers[0].wqkv, TealWeight)
    tech.detach()
    for k, v in model.state_dict().items():
        assert torch.equal(v, before[k]), k


def test_teal_phases_select_paths():
    model = tiny_model()
    eco.apply(model, TealConfig(sparsity=0.5, allocation="uniform", backend="dense"), calibration=CAL)
    w = model.layers[1].w_down
    x = torch.randn(1, 5, w.shape[1])
    dense = F.linear(x, w.dequantize())
    with phase("prefill"):
        assert torch.allclose(w.linear(x), dense)
    with phase("draft"):
        assert torch.allclose(w.linear(x), F.linear(sparsify(x, w.threshold), w.dequantize()))
    assert not torch.allclose(F.linear(sparsify(x, w.threshold), w.dequantize()), dense)


def test_teal_state_roundtrip_skips_calibration(tmp_path):
    model = tiny_model()
    eff = eco.apply(model, TealConfig(sparsity=0.3, allocation="uniform", backend="dense"), calibration=CAL)
    thr = eff.techniques["teal"].thresholds.clone()
    eff.save_pretrained(tmp_path / "m")
    again = eco.load(tiny_model(), tmp_path / "m")
    assert torch.equal(again.techniques["teal"].thresholds.cpu(), thr.cpu())


def test_teal_auto_refuses_cpu_maps():
    with pytest.raises(eco.ConfigError, match="backend='dense'"):
        eco.apply(tiny_model(), TealConfig(sparsity=0.3, allocation="uniform"), calibration=CAL)
    with pytest.raises(eco.ConfigError, match="CUDA"):
        TealConfig(backend="triton")


def test_cats_thresholds_hit_target_and_decode():
    model = tiny_model()
    eff = eco.apply(model, CatsConfig(sparsity=0.5, backend="dense"), calibration=CAL)
    tech = eff.techniques["cats"]
    assert tech.calibrated and (tech.thresholds > 0).all()
    # realised channel sparsity of the calibration pass's gate activations
    layer = model.layers[2]
    x = torch.randn(64, model.config.hidden_size) * 0.5
    f = layer.w_gate_up.shape[0] // 2
    g = F.silu(F.linear(x, layer.w_gate_up[:f]))
    assert 0.1 < float((g.abs() <= tech.thresholds[2]).float().mean()) < 0.95
    out = eff.decode(prompts((12,))[0], 5)
    assert out.tokens.numel() == 5
    tech.detach()
    assert getattr(model.layers[0], "mlp_rule", None) is None


@pytest.mark.parametrize("source", ["mlp", "lookahead"])
def test_dejavu_fit_improves_recall_and_decodes(source):
    model = tiny_model()
    cfg = DejaVuConfig(sparsity=0.5, rank=32, fit_steps=60, fit_batch=64, backend="dense", predictor_input=source)
    eff = eco.apply(model, cfg, calibration=CAL)
    tech = eff.techniques["dejavu"]
    assert bool(tech.fitted)
    out = eff.decode(prompts((12,))[0], 4)
    assert out.tokens.numel() == 4
    # the fitted predictor beats chance at recalling the dense model's top channels
    from economize_b200.techniques.mlp_sparsity import dejavu_labels

    data = tech._collect([CAL])
    a, m = data[0]
    labels = dejavu_labels(model.layers[0].w_gate_up, m, tech.k)
    pred = torch.zeros_like(labels).scatter_(-1, tech.predict(0, a).topk(tech.k, -1).indices, True)
    recall = float((pred & labels).sum() / labels.sum())
    assert recall > 0.55, recall


def test_dejavu_objective_trains():
    from economize_b200.train.objective import OBJECTIVES

    model = tiny_model()
    eff = eco.apply(model, DejaVuConfig(sparsity=0.5, rank=16, fit_steps=0, backend="dense"), calibration=CAL)
    obj = OBJECTIVES.get("dejavu")(eff)
    opt = torch.optim.Adam(obj.parameters(), lr=1e-2)
    first = None
    for _ in range(15):
        loss, _ = obj.loss(CAL)
        opt.zero_grad()
        loss.backward()
        opt.step()
        first = first if first is not None else float(loss.detach())
    assert float(loss.detach()) < first


# ---- GPU ------------------------------------------------------------------------------------------------------
@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N", [(1, 4096, 6144), (3, 4096, 1024), (8, 14336, 4096), (16, 1024, 264), (2, 128, 512)])
def test_colsparse_linear_matches_reference(cuda, M, K, N):
    from economize_b200.ops._ext import require

    g = torch.Generator(device=cuda).manual_seed(M + K)
    x = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.02).bfloat16()
    t = torch.tensor(0.6, device=cuda)
    wt = w.t().contiguous()
    out = require().colsparse_linear(x, wt, t)
    ref = F.linear(sparsify(x, t).float(), w.float())
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
    # exact zeros only (no threshold) and determinism
    xz = x.masked_fill(torch.rand(M, K, device=cuda, generator=g) < 0.5, 0)
    a = require().colsparse_linear(xz, wt, None)
    torch.testing.assert_close(a.float(), F.linear(xz.float(), w.float()), atol=2e-2, rtol=2e-2)
    assert torch.equal(a, require().colsparse_linear(xz, wt, None))


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 4, 11])
def test_glu_rows_match_reference(cuda, M):
    from economize_b200.ops._ext import require

    H, Fw = 1024, 2816
    g = torch.Generator(device=cuda).manual_seed(M)
    x = torch.randn(M, H, device=cuda, generator=g).bfloat16()
    w = (torch.randn(2 * Fw, H, device=cuda, generator=g) * 0.03).bfloat16()
    gate = F.linear(x, w[:Fw])
    t = torch.tensor(0.15, device=cuda)
    h = require().glu_rows(x, w, gate, None, t)
    s = F.silu(gate)
    up = F.linear(x, w[Fw:])
    ref = torch.where(s.abs() > t.bfloat16(), s, torch.zeros_like(s)) * up
    torch.testing.assert_close(h.float(), ref.float(), atol=1e-2, rtol=2e-2)
    assert 0.2 < float((h == 0).float().mean()) < 0.95
    keep = torch.rand(M, Fw, device=cuda, generator=g) < 0.4
    h2 = require().glu_rows(x, w, None, keep, None)
    ref2 = (F.silu(gate) * up).masked_fill(~keep, 0)
    torch.testing.assert_close(h2.float(), ref2.float(), atol=1e-2, rtol=2e-2)


@pytest.mark.gpu
def test_sparse_techniques_kernel_path_matches_masked_dense(cuda):
    from .helpers import gpu_tiny_model

    cal = torch.randint(0, 1024, (2, 64), generator=torch.Generator().manual_seed(5)).to(cuda)
    from economize_b200.runtime.cache import StepBatch

    def decode_hidden(model):
        cache = model.new_cache(1, 128)
        n = torch.tensor([9], dtype=torch.int32, device=cuda)
        model.forward_step(cal[:1, :9], StepBatch.prefill(n, 9), cache)
        one = torch.ones(1, dtype=torch.int32, device=cuda)
        sb = StepBatch(n, one, n[:, None].contiguous(), torch.ones(1, 1, dtype=torch.int64, device=cuda))
        with phase("decode"):
            return model.forward_step(cal[:1, 9:10], sb, cache)[0].float()

    for cfg_k, cfg_d in ((TealConfig(sparsity=0.4, allocation="uniform", backend="auto"),
                          TealConfig(sparsity=0.4, allocation="uniform", backend="dense")),
                         (CatsConfig(sparsity=0.5, backend="auto"), CatsConfig(sparsity=0.5, backend="dense")),
                         (DejaVuConfig(sparsity=0.5, rank=32, fit_steps=20, backend="auto"),
                          DejaVuConfig(sparsity=0.5, rank=32, fit_steps=20, backend="dense"))):
        mk = gpu_tiny_model(cuda)
        md = gpu_tiny_model(cuda)
        dense = decode_hidden(gpu_tiny_model(cuda))
        eco.apply(mk, cfg_k, calibration=cal)
        eco.apply(md, cfg_d, calibration=cal)
        hk, hd = decode_hidden(mk), decode_hidden(md)
        assert (hk - hd).abs().max() < 0.1 * hd.abs().max(), cfg_k
        assert (hd - dense).abs().max() > 0, cfg_k  # the sparsity changed something
