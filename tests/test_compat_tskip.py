"""tskip ``jump.pt`` readers: each shape is detected by exactly one format, loads into the technique it describes
with its tensors in place, and malformed or unsupported files fail with CheckpointFormatError."""

from __future__ import annotations

import pytest
import torch

import economize_b200 as eco
from economize_b200.compat import TSKIP_KINDS, cost_events
from economize_b200.core.serialization import read_checkpoint
from economize_b200.decoding.cost import CostKind, CostLog
from economize_b200.errors import CheckpointFormatError

from .helpers import tiny_model


def _medusa_file(tmp_path, heads=3, hidden=256):
    g = torch.Generator().manual_seed(3)
    raw = {"kind": "medusa", "K": heads, "model": "tiny", "state": {
        "W": torch.randn(heads, hidden, hidden, generator=g) * 0.01, "b": torch.randn(heads, hidden, generator=g)}}
    run = tmp_path / "medusa_run"
    run.mkdir()
    torch.save(raw, run / "jump.pt")
    return run, raw


def _eagle3_state(hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=688, n_aux=3, bias=False):
    g = torch.Generator().manual_seed(5)

    def r(*shape):
        return torch.randn(*shape, generator=g) * 0.02

    state = {"mix.proj.weight": r(hidden, n_aux * hidden), "pred.hidden_norm.weight": 1 + r(hidden),
             "pred.layer.input_layernorm.weight": 1 + r(hidden),
             "pred.layer.post_attention_layernorm.weight": 1 + r(hidden),
             "pred.layer.self_attn.q_proj.weight": r(heads * head_dim, 2 * hidden),
             "pred.layer.self_attn.k_proj.weight": r(kv_heads * head_dim, 2 * hidden),
             "pred.layer.self_attn.v_proj.weight": r(kv_heads * head_dim, 2 * hidden),
             "pred.layer.self_attn.o_proj.weight": r(hidden, heads * head_dim),
             "pred.layer.mlp.gate_proj.weight": r(ffn, hidden), "pred.layer.mlp.up_proj.weight": r(ffn, hidden),
             "pred.layer.mlp.down_proj.weight": r(hidden, ffn)}
    if bias:
        for n in "qkv":
            rows = state[f"pred.layer.self_attn.{n}_proj.weight"].shape[0]
            state[f"pred.layer.self_attn.{n}_proj.bias"] = r(rows)
    return state


def test_medusa_jump_pt_loads_into_shared_head_medusa(tmp_path):
    run, raw = _medusa_file(tmp_path)
    assert sorted(n for n in eco.FORMATS.names() if eco.FORMATS.get(n).detect(run)) == ["tskip_medusa"]
    ckpt = read_checkpoint(run)
    (config,) = ckpt.configs
    assert (config.num_heads, config.num_layers, config.head) == (3, 1, "shared")
    assert ckpt.base_model == "tiny"
    em = eco.load(tiny_model(), run)
    tech = em.techniques["medusa"]
    for k in range(3):
        torch.testing.assert_close(tech.heads[k].blocks[0].linear.weight.float(), raw["state"]["W"][k])
        torch.testing.assert_close(tech.heads[k].blocks[0].linear.bias.float(), raw["state"]["b"][k])
    out = em.generate(torch.arange(5)[None], max_new_tokens=4)
    assert out.shape[-1] >= 9


def test_eagle3_jump_pt_loads_with_model_head_and_fused_sources(tmp_path):
    from economize_b200.techniques.eagle3.formats import to_reference_state

    state = _eagle3_state()
    raw = {"cfg": {"pred": "eagle3", "feed": "fused", "mix": "fc", "m": 4, "u": 4, "r": 4, "src": "1,2,3"},
           "model": "tiny", "state": state}
    file = tmp_path / "e3.pt"
    torch.save(raw, file)
    assert [n for n in eco.FORMATS.names() if eco.FORMATS.get(n).detect(file)] == ["tskip_eagle3"]
    ckpt = read_checkpoint(file)
    (config,) = ckpt.configs
    assert config.aux_layers == (1, 2, 3) and config.head == "shared" and config.zero_source_first
    em = eco.load(tiny_model(), file)
    got = to_reference_state(em.techniques["eagle3"])
    torch.testing.assert_close(got["fc.weight"], state["mix.proj.weight"])
    for key, value in state.items():
        if key.startswith("pred.layer."):
            torch.testing.assert_close(got["layer." + key[len("pred.layer."):]], value)
    torch.testing.assert_close(got["layer.hidden_norm.weight"], state["pred.hidden_norm.weight"])
    assert "lm_head.weight" not in got  # the model's own head drafts


def test_eagle3_jump_pt_with_bias_and_bad_layouts(tmp_path):
    base = {"pred": "eagle3", "feed": "fused", "mix": "fc", "m": 4, "u": 4, "r": 4, "src": "1,2,3"}
    file = tmp_path / "bias.pt"
    torch.save({"cfg": base, "state": _eagle3_state(bias=True)}, file)
    assert read_checkpoint(file).configs[0].attention_bias
    for cfg, why in (({**base, "r": 3}, "m = u = r"), ({**base, "mode": "lora"}, "frozen"),
                     ({**base, "src": "1,2"}, "fuses 2 layers")):
        bad = tmp_path / "bad.pt"
        torch.save({"cfg": cfg, "state": _eagle3_state()}, bad)
        with pytest.raises(CheckpointFormatError, match=why):
            read_checkpoint(bad)
    state = _eagle3_state()
    state["pred.layer.self_attn.q_norm.weight"] = torch.ones(64)
    torch.save({"cfg": base, "state": state}, tmp_path / "qn.pt")
    with pytest.raises(CheckpointFormatError, match="q/k norms"):
        read_checkpoint(tmp_path / "qn.pt")


def test_medusa_and_jump_refusals(tmp_path):
    run = tmp_path / "m"
    run.mkdir()
    torch.save({"kind": "medusa", "K": 2, "state": {"W": torch.zeros(2, 8, 8)}}, run / "jump.pt")
    with pytest.raises(CheckpointFormatError, match="exactly 'W' and 'b'"):
        read_checkpoint(run)
    torch.save({"kind": "medusa", "K": 3, "state": {"W": torch.zeros(2, 8, 8), "b": torch.zeros(2, 8)}},
               run / "jump.pt")
    with pytest.raises(CheckpointFormatError, match="K=3"):
        read_checkpoint(run)
    jump = tmp_path / "jump.pt"
    torch.save({"cfg": {"pred": "mlp", "m": 2, "u": 3, "r": 4}, "state": {"pred.ps.weight": torch.zeros(4, 4)}},
               jump)
    assert [n for n in eco.FORMATS.names() if eco.FORMATS.get(n).detect(jump)] == ["tskip"]
    with pytest.raises(CheckpointFormatError, match="jump technique"):
        read_checkpoint(jump)


def test_unreadable_and_foreign_files_are_not_tskip(tmp_path):
    (tmp_path / "junk.pt").write_bytes(b"not a zip archive")
    torch.save([torch.zeros(2)], tmp_path / "list.pt")
    for name in ("junk.pt", "list.pt"):
        assert not any(eco.FORMATS.get(n).detect(tmp_path / name) for n in ("tskip", "tskip_eagle3", "tskip_medusa"))


def test_cost_events_use_tskip_names():
    log = CostLog()
    log.record(CostKind.EXACT, 12, 0, 0, 3)
    log.record(CostKind.DRAFT, 1, 12, 0, 1)
    log.record(CostKind.DRAFT_WASTED, 1, 13, 0, 1)
    log.record(CostKind.DRAFT_OBSERVE, 2, 12, 0, 0)
    log.record(CostKind.REPLAY, 1, 14, 0, 3)
    assert cost_events(log) == [("exact", 12, 0), ("jump", 1, 12), ("jump_wasted", 1, 13), ("pred_ctx", 2, 12),
                                (CostKind.REPLAY, 1, 14)]
    assert set(TSKIP_KINDS) <= {CostKind.EXACT, CostKind.DRAFT, CostKind.DRAFT_WASTED, CostKind.DRAFT_OBSERVE}
