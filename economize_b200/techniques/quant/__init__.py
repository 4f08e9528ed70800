"""Weight quantization: ``quant`` (RTN / GPTQ / AWQ of the target, int4 / int8 / fp8 weights) and
``draft_quant`` (round-to-nearest of the drafter only), executed by the tcgen05 weight-only GEMM."""

from .config import QUANT_FORMATS, DraftQuantConfig, QuantConfig
from .methods import awq_clip, awq_search, gptq, rtn
from .technique import DraftQuantTechnique, QuantTechnique

__all__ = ["DraftQuantConfig", "DraftQuantTechnique", "QUANT_FORMATS", "QuantConfig", "QuantTechnique", "awq_clip",
           "awq_search", "gptq", "rtn"]
