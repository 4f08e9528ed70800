"""Benchmark utilities: device timing (:mod:`.timing`), the analytic cost model with a B200 preset
(:mod:`.cost_model`), kernel micro-benchmarks (``python -m economize_b200.bench.kernels``) and prompt sets
(:mod:`.prompts`)."""

from .cost_model import HARDWARE, Hardware, decode_step_cost, roofline
from .timing import Timing, max_over_ranks, time_call

__all__ = ["HARDWARE", "Hardware", "Timing", "decode_step_cost", "max_over_ranks", "roofline", "time_call"]
