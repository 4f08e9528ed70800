"""Integrations with other tools' file formats (economize ``src/economize/integrations``):
:mod:`~economize_b200.integrations.compressed_tensors` writes quantized targets for llm-compressor's loaders,
:mod:`~economize_b200.integrations.peft` reads and writes LoRA adapters in PEFT's format,
:mod:`~economize_b200.integrations.lm_eval` runs lm-evaluation-harness requests through an efficient model."""
