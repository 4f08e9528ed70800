"""Writing trained techniques out for other inference engines (economize ``src/economize/backends``).

* :func:`export_drafter`: a drafter technique as the draft-model folder (``config.json`` + ``model.safetensors``)
  that one serving engine loads; exporters are registered per ``"<backend>/<technique>"`` in :data:`EXPORTERS`
  (built in: ``vllm/eagle3``, ``vllm/eagle``, ``vllm/medusa``, ``sglang/eagle3``, ``sglang/eagle``).
* :func:`to_gguf`: the target model (with any weight transform folded in) as one GGUF file for llama.cpp-style
  runtimes, in F32, F16, BF16 or Q8_0; :func:`read_gguf` reads such a file back.

These only write files: the engines themselves are not imported, and nothing here runs on the decoding path.
"""

from __future__ import annotations

from .exporters import (EXPORTERS, DrafterExporter, UnsupportedBackendError, export_drafter, exporter_for,
                        register_exporter)
from .gguf import GGUF_TYPES, read_gguf, to_gguf

from . import sglang, vllm  # noqa: E402,F401  (register the built-in exporters)

__all__ = ["EXPORTERS", "GGUF_TYPES", "DrafterExporter", "UnsupportedBackendError", "export_drafter",
           "exporter_for", "read_gguf", "register_exporter", "to_gguf"]
