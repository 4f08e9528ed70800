"""Checkpoints of the ``tskip`` research code (``jump.pt``) and its cost-log naming.

``tskip`` (the research predecessor of economize) stores each trained drafter as a single ``torch.save`` dict called
``jump.pt`` (economize ``compat/tskip.py:1-16``). Three shapes of that dict exist:

* ``{"kind": "medusa", "K": heads, "model": base, "state": {"W": [K, d, d], "b": [K, d]}}``: Medusa heads with one
  residual block each and the model's own norm and LM head. Read as :class:`~..techniques.medusa.MedusaConfig`
  (``num_layers=1``, ``head="shared"``); head ``k``'s block gets ``W[k]``, ``b[k]``.
* ``{"cfg": {..., "pred": "eagle3", "feed": "fused", "mix": "fc", "m" = "u" = "r", "src": "2,16,29"}, "state"}``:
  an EAGLE-3 layer whose fusion matrix is ``mix.proj``, whose decoder layer is ``pred.layer.*`` (HF names) and
  whose norm/head are the model's. Read as :class:`~..techniques.eagle3.Eagle3Config` (``head="shared"``, the
  first position drafting from a zero source, attention bias when the state has one).
* any other ``{"cfg", "state"}`` dict: a jump drafter. Its block predictors, readouts and source mixers have module
  layouts that this package's jump technique does not build; reading one raises a
  :class:`~..errors.CheckpointFormatError` that says so, instead of loading a partial drafter.

The three shapes are told apart by the dict alone (``kind == "medusa"``, ``cfg["pred"] == "eagle3"``, else jump),
so each registered format accepts exactly one of them and detection is unambiguous. A file is loaded with
``weights_only=True`` (plain tensors and containers; no code runs) and memory-mapped while probing.

:func:`cost_events` renames a :class:`~..decoding.cost.CostLog` to tskip's event names so per-call logs of the two
decoders can be compared.
"""

from __future__ import annotations

import logging
import pickle
from collections.abc import Mapping
from pathlib import Path
from typing import Any

import torch

from ..core.serialization import FORMATS, Checkpoint, CheckpointFormat
from ..decoding.cost import CostKind, CostLog
from ..errors import CheckpointFormatError, ConfigError

__all__ = ["TSKIP_EAGLE3", "TSKIP_JUMP", "TSKIP_KINDS", "TSKIP_MEDUSA", "TskipEagle3Format", "TskipJumpFormat",
           "TskipMedusaFormat", "cost_events", "eagle3_from_tskip", "medusa_from_tskip", "tskip_kind"]

logger = logging.getLogger(__name__)

TSKIP_JUMP, TSKIP_EAGLE3, TSKIP_MEDUSA = "jump", "eagle3", "medusa"

#: this package's cost kinds under tskip's names (economize ``compat/tskip.py:76-82``); kinds tskip never logs keep
#: their own names
TSKIP_KINDS: Mapping[str, str] = {
    CostKind.EXACT: "exact",
    CostKind.DRAFT: "jump",
    CostKind.DRAFT_WASTED: "jump_wasted",
    CostKind.DRAFT_OBSERVE: "pred_ctx",
}


def cost_events(log: CostLog) -> list[tuple[str, int, int]]:
    """``(kind, tokens, position)`` of every event of ``log`` under tskip's kind names, in logging order."""
    return log.as_tuples(TSKIP_KINDS)


def _file(path: str | Path) -> Path:
    path = Path(path)
    return path if path.suffix == ".pt" else path / "jump.pt"


def _load(path: str | Path, mmap: bool) -> dict[str, Any] | None:
    """The ``jump.pt`` dict at ``path`` (a ``.pt`` file or a run directory), or ``None`` when there is none or it
    is not a tskip dict (anything ``torch.load`` refuses counts as not a tskip file, with a logged warning)."""
    file = _file(path)
    if not file.is_file():
        return None
    try:
        raw = torch.load(file, map_location="cpu", mmap=mmap, weights_only=True)
    except (OSError, RuntimeError, EOFError, pickle.UnpicklingError) as error:
        logger.warning("economize_b200: %s is not a readable tskip checkpoint (%s: %s)", file,
                       type(error).__name__, error)
        return None
    return raw if isinstance(raw, dict) and "state" in raw else None


def tskip_kind(raw: Mapping[str, Any]) -> str:
    """Which of the three ``jump.pt`` shapes ``raw`` is (the module docstring lists them)."""
    if raw.get("kind") == "medusa":
        return TSKIP_MEDUSA
    cfg = raw.get("cfg")
    if isinstance(cfg, Mapping) and cfg.get("pred") == "eagle3":
        return TSKIP_EAGLE3
    return TSKIP_JUMP


def medusa_from_tskip(raw: Mapping[str, Any]) -> Checkpoint:
    """The checkpoint of a Medusa ``jump.pt``: one residual block per head over the model's norm and LM head."""
    from ..techniques.medusa import MedusaConfig

    state = raw.get("state")
    if not isinstance(state, Mapping) or set(state) != {"W", "b"}:
        got = sorted(state) if isinstance(state, Mapping) else type(state).__name__
        raise CheckpointFormatError(f"a Medusa jump.pt state holds exactly 'W' and 'b', got {got}")
    weight, bias = state["W"], state["b"]
    if weight.dim() != 3 or weight.shape[1] != weight.shape[2] or tuple(bias.shape) != tuple(weight.shape[:2]):
        raise CheckpointFormatError(f"Medusa jump.pt shapes W {tuple(weight.shape)} and b {tuple(bias.shape)} are "
                                    "not [K, d, d] and [K, d]")
    heads = int(raw.get("K", weight.shape[0]))
    if heads != weight.shape[0]:
        raise CheckpointFormatError(f"Medusa jump.pt says K={heads} but stores {weight.shape[0]} heads")
    tensors: dict[str, torch.Tensor] = {}
    for k in range(heads):
        tensors[f"heads.{k}.blocks.0.linear.weight"] = weight[k].clone()
        tensors[f"heads.{k}.blocks.0.linear.bias"] = bias[k].clone()
    try:
        config = MedusaConfig(num_heads=heads, num_layers=1, head="shared")
    except ConfigError as error:
        raise CheckpointFormatError(f"invalid Medusa jump.pt: {error}") from error
    return Checkpoint([config], {"medusa": tensors}, None, raw.get("model"), {"format": "tskip_medusa"})


def _layers(src: Any, fallback: Any) -> tuple[int, ...]:
    text = str(src) if src not in (None, "") else str(fallback)
    try:
        return tuple(sorted({int(part) for part in text.split(",") if part.strip()}))
    except ValueError as error:
        raise CheckpointFormatError(f"EAGLE-3 jump.pt src={src!r} is not a comma-separated list of layers") from error


def eagle3_from_tskip(raw: Mapping[str, Any]) -> Checkpoint:
    """The checkpoint of an EAGLE-3 ``jump.pt``: fused sources ``src`` (the exit layer when absent), the model's
    norm and LM head, a zero source at the first drafted position."""
    from ..techniques.eagle3 import Eagle3Config

    cfg = raw.get("cfg")
    if not isinstance(cfg, Mapping) or cfg.get("pred") != "eagle3":
        raise CheckpointFormatError("not an EAGLE-3 jump.pt (its cfg['pred'] is not 'eagle3')")
    exits = {cfg.get("m"), cfg.get("u"), cfg.get("r")}
    if cfg.get("feed") != "fused" or cfg.get("mix") != "fc" or len(exits) != 1:
        raise CheckpointFormatError("an EAGLE-3 jump.pt needs feed='fused', mix='fc' and m = u = r; got "
                                    f"feed={cfg.get('feed')!r} mix={cfg.get('mix')!r} m/u/r={sorted(map(str, exits))}")
    if cfg.get("mode", "frozen") != "frozen":
        raise CheckpointFormatError(f"EAGLE-3 jump.pt in mode {cfg.get('mode')!r}: only frozen targets are read")
    state = raw["state"]
    tensors: dict[str, torch.Tensor] = {}
    for key, value in state.items():
        if key == "mix.proj.weight":
            tensors["fc.weight"] = value
        elif key == "pred.hidden_norm.weight":
            tensors["layer.hidden_norm.weight"] = value
        elif key.startswith("pred.layer."):
            leaf = key.split(".", 2)[2]
            if leaf.startswith(("self_attn.q_norm", "self_attn.k_norm")):
                raise CheckpointFormatError(f"EAGLE-3 jump.pt layers with q/k norms are not read ({key!r})")
            tensors["layer." + leaf] = value
        else:
            raise CheckpointFormatError(f"unexpected parameter {key!r} in an EAGLE-3 jump.pt")
    needed = {"fc.weight", "layer.input_layernorm.weight", "layer.hidden_norm.weight",
              "layer.self_attn.q_proj.weight", "layer.mlp.down_proj.weight"}
    if needed - set(tensors):
        raise CheckpointFormatError(f"EAGLE-3 jump.pt lacks {sorted(needed - set(tensors))}")
    aux = _layers(cfg.get("src"), cfg.get("u"))
    if tensors["fc.weight"].shape[1] != len(aux) * tensors["fc.weight"].shape[0]:
        raise CheckpointFormatError(f"EAGLE-3 jump.pt fuses {len(aux)} layers {aux} but its fc weight is "
                                    f"{tuple(tensors['fc.weight'].shape)}")
    try:
        config = Eagle3Config(aux_layers=aux, head="shared", zero_source_first=True,
                              attention_bias="layer.self_attn.q_proj.bias" in tensors)
    except ConfigError as error:
        raise CheckpointFormatError(f"invalid EAGLE-3 jump.pt: {error}") from error
    return Checkpoint([config], {"eagle3": tensors}, None, raw.get("model"), {"format": "tskip_eagle3"})


class _TskipFormat(CheckpointFormat):
    """One of the three ``jump.pt`` shapes: detection loads the dict memory-mapped and checks its shape."""

    kind: str

    def detect(self, path: Path) -> bool:
        raw = _load(path, mmap=True)
        return raw is not None and tskip_kind(raw) == self.kind

    def read(self, path: Path) -> Checkpoint:
        raw = _load(path, mmap=False)
        if raw is None:
            raise CheckpointFormatError(f"{_file(path)} is not a tskip jump.pt (a dict with a 'state')")
        if tskip_kind(raw) != self.kind:
            raise CheckpointFormatError(f"{_file(path)} is a tskip {tskip_kind(raw)} checkpoint, not {self.kind}")
        try:
            checkpoint = self.convert(raw)
        except CheckpointFormatError as error:
            raise CheckpointFormatError(f"{_file(path)}: {error}") from error
        checkpoint.meta.setdefault("source", str(_file(path)))
        return checkpoint

    def convert(self, raw: Mapping[str, Any]) -> Checkpoint:
        raise NotImplementedError


class TskipMedusaFormat(_TskipFormat):
    kind = TSKIP_MEDUSA

    def convert(self, raw: Mapping[str, Any]) -> Checkpoint:
        return medusa_from_tskip(raw)


class TskipEagle3Format(_TskipFormat):
    kind = TSKIP_EAGLE3

    def convert(self, raw: Mapping[str, Any]) -> Checkpoint:
        return eagle3_from_tskip(raw)


class TskipJumpFormat(_TskipFormat):
    """Recognises tskip jump drafters so that ``load`` names them, and refuses to read them: their predictor,
    readout and mixer modules have no counterpart in this package's jump technique."""

    kind = TSKIP_JUMP

    def convert(self, raw: Mapping[str, Any]) -> Checkpoint:
        cfg = raw.get("cfg") if isinstance(raw.get("cfg"), Mapping) else {}
        raise CheckpointFormatError(
            f"tskip jump drafters (pred={cfg.get('pred', 'mlp')!r}, m/u/r={cfg.get('m')}/{cfg.get('u')}/"
            f"{cfg.get('r')}) use block predictors, readouts and source mixers that economize_b200's jump technique "
            "does not build; retrain with economize_b200.train.fit and JumpConfig")


for _name, _format in (("tskip", TskipJumpFormat()), ("tskip_eagle3", TskipEagle3Format()),
                       ("tskip_medusa", TskipMedusaFormat())):
    if _name not in FORMATS:
        FORMATS.register(_name, _format)
