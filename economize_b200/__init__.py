"""economize_b200: a Blackwell-native (B200, sm_100a) framework for composable LLM-inference efficiency.

    import economize_b200 as economize
    from economize_b200.techniques.eagle3 import Eagle3Config

    model = economize.apply(hf_model, Eagle3Config())
    out = model.generate(input_ids, max_new_tokens=128,
                         decoding=economize.DecodeConfig(cycle_length=7, draft_policy="dynamic_tree",
                                                         draft_policy_options={"depth": 6, "topk": 10,
                                                                               "total_tokens": 60},
                                                         cuda_graphs=True))

The public surface mirrors economize 0.6 (``src/economize/__init__.py``): ``apply``, ``EfficientModel``,
``DecodeConfig``, the technique configs under ``economize_b200.techniques.<name>``, the error classes, ``save`` /
``load`` / ``from_pretrained``. Execution is the engine's own: fused Llama-family executor, tcgen05/TMA kernels,
one CUDA graph per speculative cycle.
"""

from __future__ import annotations

from . import techniques  # noqa: F401  (registers the built-in techniques)
from ._version import API_LEVEL, __version__
from .core import CAPABILITY_ORDER, TECHNIQUES, Capability, Family, Simulation, Technique, TechniqueConfig, \
    register_technique, technique_for
from .core.compatibility import compatibility_matrix, compatible, incompatibility, listed_techniques
from .core.model import EfficientModel, apply, build_model
from .core.serialization import (FORMATS, Checkpoint, CheckpointFormat, attach, from_pretrained, load,
                                 read_checkpoint, save, teacher_fingerprint)
from .decoding import DecodeConfig, DecodeResult, GreedySelector, SpecEngine, TokenSelector, TopPSampler
from . import ops  # noqa: F401
from . import compat  # noqa: F401  (registers the tskip checkpoint formats)
from .errors import (CalibrationMismatchWarning, CheckpointFormatError, CommTimeoutError, ConfigError,
                     DuplicateNameError, EconomizeError, IncompatibleTechniquesError, KernelUnavailableError,
                     NonFiniteLossError, SimulatedPathWarning, TeacherMismatchWarning, UnknownFieldWarning,
                     UnknownNameError, UnregisteredNameError, UnsupportedEngineVersionError, UnsupportedModelError,
                     UntestedEngineWarning)

__all__ = [
    "API_LEVEL", "CAPABILITY_ORDER", "FORMATS", "TECHNIQUES", "Checkpoint", "CheckpointFormat", "attach",
    "compatibility_matrix", "compatible", "from_pretrained", "incompatibility", "listed_techniques", "load",
    "read_checkpoint", "save", "teacher_fingerprint", "CalibrationMismatchWarning", "Capability",
    "CheckpointFormatError", "CommTimeoutError", "ConfigError", "DecodeConfig", "DecodeResult", "DuplicateNameError",
    "EconomizeError", "EfficientModel", "Family", "GreedySelector", "IncompatibleTechniquesError",
    "KernelUnavailableError", "NonFiniteLossError", "SimulatedPathWarning", "Simulation", "SpecEngine", "Technique",
    "TechniqueConfig", "TeacherMismatchWarning", "TokenSelector", "TopPSampler", "UnknownFieldWarning",
    "UnknownNameError", "UnregisteredNameError", "UnsupportedEngineVersionError", "UnsupportedModelError",
    "UntestedEngineWarning", "__version__", "apply", "build_model", "register_technique", "technique_for",
]
