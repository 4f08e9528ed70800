"""Readers for checkpoints of other codebases (economize ``compat/``): importing this package registers their
formats in :data:`economize_b200.FORMATS`."""

from .tskip import (TSKIP_EAGLE3, TSKIP_JUMP, TSKIP_KINDS, TSKIP_MEDUSA, TskipEagle3Format, TskipJumpFormat,
                    TskipMedusaFormat, cost_events, eagle3_from_tskip, medusa_from_tskip, tskip_kind)

__all__ = ["TSKIP_EAGLE3", "TSKIP_JUMP", "TSKIP_KINDS", "TSKIP_MEDUSA", "TskipEagle3Format", "TskipJumpFormat",
           "TskipMedusaFormat", "cost_events", "eagle3_from_tskip", "medusa_from_tskip", "tskip_kind"]
