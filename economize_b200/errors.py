"""Exception and warning classes.

The class names and their base classes mirror economize (``src/economize/errors.py:24-96``) so that code written
against economize catches the same errors here: a ``ConfigError`` is also a ``ValueError``, an unknown registry name
is also a ``KeyError``, and so on.
"""

from __future__ import annotations

__all__ = [
    "CalibrationMismatchWarning",
    "CheckpointFormatError",
    "CommTimeoutError",
    "ConfigError",
    "DuplicateNameError",
    "EconomizeError",
    "IncompatibleTechniquesError",
    "KernelUnavailableError",
    "NonFiniteLossError",
    "SimulatedPathWarning",
    "TeacherMismatchWarning",
    "UnknownFieldWarning",
    "UnknownNameError",
    "UnregisteredNameError",
    "UnsupportedEngineVersionError",
    "UnsupportedModelError",
    "UntestedEngineWarning",
]


class EconomizeError(Exception):
    """Root of every error this package raises on purpose."""


class ConfigError(EconomizeError, ValueError):
    """An option is invalid on its own or for the model it is applied to."""


class UnknownNameError(EconomizeError, KeyError):
    """A name is missing from a registry; the message lists what is registered."""

    def __str__(self) -> str:
        return str(self.args[0]) if self.args else ""


class UnregisteredNameError(ConfigError, UnknownNameError):
    """A configuration field names a registry entry that does not exist."""


class DuplicateNameError(EconomizeError, ValueError):
    """A registry name was taken already and ``override`` was not given."""


class UnsupportedModelError(EconomizeError, TypeError):
    """The model's architecture or layout is not one this package can execute."""


class IncompatibleTechniquesError(EconomizeError, ValueError):
    """Two techniques cannot be attached to the same model."""


class CheckpointFormatError(EconomizeError, ValueError):
    """A checkpoint has an unknown layout or does not fit its configuration."""


class NonFiniteLossError(EconomizeError, FloatingPointError):
    """A training loss was NaN or infinite and the run is configured to stop on it."""


class UnsupportedEngineVersionError(EconomizeError, ImportError):
    """An external serving engine is missing or outside the tested version range."""


class KernelUnavailableError(EconomizeError, RuntimeError):
    """A CUDA tensor reached an operator whose compiled sm_100a extension is not loaded.

    CUDA inputs never fall back to a PyTorch implementation silently: build the extension
    (``python setup.py build_ext --inplace`` or ``__graft_entry__.build()``) and retry.
    """


class CommTimeoutError(EconomizeError, TimeoutError):
    """A bounded device-side wait on a peer GPU (a fused collective's flag) ran out; the kernel returned early and
    reported it through its status word instead of hanging the GPU."""


class UntestedEngineWarning(UserWarning):
    """An engine release outside the tested range is used because the user allowed it."""


class SimulatedPathWarning(UserWarning):
    """A technique runs on a path that reproduces its outputs but not its savings (e.g. fake quantization)."""


class CalibrationMismatchWarning(UserWarning):
    """Replaying a checkpoint's weight techniques gave other weights than the saved ones (other calibration data)."""


class UnknownFieldWarning(UserWarning):
    """A saved configuration holds fields this version does not know; they are dropped."""


class TeacherMismatchWarning(UserWarning):
    """The base weights differ from those a checkpoint was trained against."""
