"""Core of the framework: technique model, the :class:`EfficientModel` facade, serialization."""

from .technique import (CAPABILITY_ORDER, TECHNIQUES, Capability, Family, Simulation, Technique, TechniqueConfig,
                        register_technique, technique_for)

__all__ = ["CAPABILITY_ORDER", "TECHNIQUES", "Capability", "Family", "Simulation", "Technique", "TechniqueConfig",
           "register_technique", "technique_for"]
