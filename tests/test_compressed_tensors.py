"""compressed-tensors export (economize ``tests/integrations/test_compressed_tensors.py``): every quant format's
codes, scales and zero points survive the trip, so the folder decodes to exactly the weights the quantized model
runs, and a model loaded from those weights decodes the same tokens."""

import json

import pytest
import torch

import economize_b200 as eco
from economize_b200.errors import ConfigError
from economize_b200.integrations.compressed_tensors import export_compressed_tensors, read_compressed_tensors
from economize_b200.models.hf import load_hf_state
from economize_b200.techniques.quant import QuantConfig

from .helpers import prompts, reference_greedy, tiny_model


@pytest.mark.parametrize("fmt,sym,ct", [("int4", False, "pack-quantized"), ("int4", True, "pack-quantized"),
                                        ("int3", False, "pack-quantized"), ("int2", False, "pack-quantized"),
                                        ("int8", True, "int-quantized"), ("fp8", True, "float-quantized"),
                                        ("mxfp4", True, "mxfp4-pack-quantized"),
                                        ("nvfp4", True, "nvfp4-pack-quantized")])
def test_roundtrip(tmp_path, fmt, sym, ct):
    eff = eco.apply(tiny_model(), QuantConfig(format=fmt, symmetric=sym, group_size=128))
    out = export_compressed_tensors(eff, tmp_path / "ct")
    config, dense = read_compressed_tensors(out)
    qc = config["quantization_config"]
    assert qc["format"] == ct and qc["quant_method"] == "compressed-tensors"
    assert qc["config_groups"]["group_0"]["weights"]["symmetric"] == (sym or fmt not in ("int2", "int3", "int4"))
    mine = eff.model.hf_state_dict()
    assert set(dense) == set(mine)
    for name, w in mine.items():
        assert torch.equal(dense[name].float(), w.float()), name
    fresh = tiny_model(seed=5)
    load_hf_state(fresh, dense)
    p = prompts((17,))[0]
    assert torch.equal(reference_greedy(fresh, p, 6), reference_greedy(eff.model, p, 6))


def test_packing_and_refusals(tmp_path):
    from economize_b200.integrations.compressed_tensors import _pack_int32, _unpack_int32

    q = torch.arange(-8, 8).repeat(3, 2)
    words = _pack_int32(q, 4)
    assert words.shape == (3, 4) and words.dtype == torch.int32
    assert words[0, 0].item() & 0xF == 0 and (words[0, 0].item() >> 28) & 0xF == 7  # -8 -> 0 first, -1 -> 7 last
    assert torch.equal(_unpack_int32(words, 4, 32), q)
    with pytest.raises(ConfigError, match="no quantized"):
        export_compressed_tensors(tiny_model(), tmp_path / "x")
    eff = eco.apply(tiny_model(), QuantConfig(format="int4", group_size=128))
    cfg = json.loads((export_compressed_tensors(eff, tmp_path / "y") / "config.json").read_text())
    ignore = cfg["quantization_config"]["ignore"]
    assert ignore[0] == "lm_head"
    unquantized = [f"model.layers.{i}.mlp.down_proj" for i in range(4)]  # 688 inputs: no 128-wide groups
    assert ignore[1:] == unquantized
