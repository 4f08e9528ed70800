"""Built-in techniques; importing this package registers every subpackage that imports cleanly."""

from ..registry import import_submodules

#: subpackages that failed to import (name -> reason)
UNAVAILABLE: dict[str, str] = {}
LOADED = import_submodules(__name__, __path__, unavailable=UNAVAILABLE)
