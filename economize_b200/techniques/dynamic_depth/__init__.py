"""Dynamic depth (economize ``techniques/dynamic_depth``): per-token layer skipping and early exit on the exact path
(``gateskip``, ``mod``, ``flexidepth``, ``skipdecode``, ``loradrop``, ``calm``; :mod:`.methods`) and the methods
that decode through the drafting cycle (``free``, ``dmtd``, ``hidden_transfer``; :mod:`.drafters`). Objectives:
``gateskip``, ``mod``, ``flexidepth``, ``loradrop``, ``calm`` (:mod:`.objectives`) and ``hidden_transfer_kl``."""

from . import objectives as _objectives  # noqa: F401  (registers the objectives)
from .base import DepthMeter, DepthPolicy, DepthTechnique, LayeredDepthConfig, ScalarScore
from .calibration import (beta_moments, bmm_threshold, calibrate_threshold, free_calibration_pairs,
                          hoeffding_bentkus_pvalue, ltt_threshold, token_mismatch)
from .drafters import (DmtdConfig, DmtdTechnique, FreeConfig, FreeTechnique, HiddenTransferConfig,
                       HiddenTransferTechnique)
from .methods import (CalmConfig, CalmTechnique, FlexiDepthConfig, FlexiDepthTechnique, GateSkipConfig,
                      GateSkipTechnique, LoRADropConfig, LoRADropTechnique, MoDConfig, MoDTechnique, SkipDecodeConfig,
                      SkipDecodeTechnique, redundant_layers)

__all__ = ["beta_moments", "bmm_threshold", "free_calibration_pairs", "calibrate_threshold", "hoeffding_bentkus_pvalue", "ltt_threshold", "token_mismatch", "CalmConfig", "CalmTechnique", "DepthMeter", "DepthPolicy", "DepthTechnique", "DmtdConfig", "DmtdTechnique",
           "FlexiDepthConfig", "FlexiDepthTechnique", "FreeConfig", "FreeTechnique", "GateSkipConfig",
           "GateSkipTechnique", "HiddenTransferConfig", "HiddenTransferTechnique", "LayeredDepthConfig",
           "LoRADropConfig", "LoRADropTechnique", "MoDConfig", "MoDTechnique", "ScalarScore", "SkipDecodeConfig",
           "SkipDecodeTechnique", "redundant_layers"]
