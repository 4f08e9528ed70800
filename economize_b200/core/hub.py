"""Hugging Face Hub persistence of an :class:`~economize_b200.core.model.EfficientModel` (economize
``core/hub.py:124-358``).

A Hub checkpoint is this package's own format (``economize_config.json`` + technique tensors, see
:mod:`economize_b200.core.serialization`) plus a ``README.md`` model card. The base model stays in its own
repository, as with a PEFT adapter: the card names it in its ``base_model:`` metadata so that the Hub links the two,
and :func:`from_pretrained` loads it from there unless a module is passed.

* :func:`model_card`: the card's text (YAML metadata, the techniques with their configurations, the decoding
  options, how to load it).
* :func:`save_pretrained`: the checkpoint and its card in a folder.
* :func:`push_to_hub`: :func:`save_pretrained` into a temporary folder, then one upload of it.
* :func:`from_pretrained`: a local folder, or a Hub repository downloaded first, attached to its base model.

The Hub calls go through ``huggingface_hub`` (``HfApi.create_repo``/``upload_folder`` and ``snapshot_download``);
the ``api`` / ``download`` arguments replace them, which is how the tests run without a network.
"""

from __future__ import annotations

import json
import tempfile
from collections.abc import Callable
from dataclasses import asdict, is_dataclass
from pathlib import Path
from typing import Any

from .._version import __version__
from ..errors import CheckpointFormatError

__all__ = ["from_pretrained", "model_card", "push_to_hub", "save_pretrained"]


def _base_name(model) -> str | None:
    base = getattr(model, "base_model", None)
    return getattr(getattr(base, "config", None), "_name_or_path", None) or None


def model_card(model, repo_id: str | None = None, base_model: str | None = None) -> str:
    """The Markdown model card of ``model``'s checkpoint."""
    base = base_model or _base_name(model)
    names = list(model.techniques.keys())
    meta = ["---", "library_name: economize_b200", "tags:", "- economize", "- speculative-decoding"]
    meta += [f"- {n}" for n in names]
    if base:
        meta.append(f"base_model: {base}")
    meta.append("---")
    lines = ["", f"# {repo_id or 'economize_b200 checkpoint'}", "",
             f"Techniques attached to {'`' + base + '`' if base else 'the base model'} with economize_b200 "
             f"{__version__}:", ""]
    for name in names:
        cfg = model.techniques[name].config
        fields = asdict(cfg) if is_dataclass(cfg) else {}
        lines.append(f"- `{name}`: `{json.dumps(fields, default=str, sort_keys=True)}`")
    decoding = getattr(model, "decoding", None)
    if decoding is not None and hasattr(decoding, "to_dict"):
        lines += ["", "Decoding options:", "", f"`{json.dumps(decoding.to_dict(), default=str, sort_keys=True)}`"]
    lines += ["", "Load with:", "", "```python", "from economize_b200.core.hub import from_pretrained", "",
              f"model = from_pretrained({(repo_id or 'path')!r}" + ("" if base else ", base_model=...") + ")", "```", ""]
    return "\n".join(meta + lines)


def save_pretrained(model, path: str | Path, *, repo_id: str | None = None, base_model: str | None = None) -> Path:
    """Write the checkpoint of ``model`` and its model card to ``path``."""
    from .serialization import save

    out = Path(path)
    save(model, out, extra_meta={"base_model": base_model} if base_model else None)
    (out / "README.md").write_text(model_card(model, repo_id, base_model))
    return out


def push_to_hub(model, repo_id: str, *, private: bool = False, token: str | None = None,
                commit_message: str = "Upload economize_b200 checkpoint", base_model: str | None = None,
                api: Any = None) -> Any:
    """Create ``repo_id`` (if needed) and upload the checkpoint; returns the upload's result."""
    if api is None:
        from huggingface_hub import HfApi

        api = HfApi(token=token)
    api.create_repo(repo_id, private=private, exist_ok=True)
    with tempfile.TemporaryDirectory() as tmp:
        save_pretrained(model, tmp, repo_id=repo_id, base_model=base_model)
        return api.upload_folder(repo_id=repo_id, folder_path=tmp, commit_message=commit_message)


def from_pretrained(repo_or_path: str | Path, base_model: Any = None, *, revision: str | None = None,
                    download: Callable[..., str] | None = None, **kwargs: Any):
    """An EfficientModel from a local checkpoint folder or a Hub repository id (downloaded with
    ``snapshot_download``); ``base_model`` as in :func:`economize_b200.core.serialization.from_pretrained`."""
    from .serialization import from_pretrained as load_folder

    path = Path(repo_or_path)
    if not path.is_dir():
        if download is None:
            from huggingface_hub import snapshot_download as download
        try:
            path = Path(download(repo_id=str(repo_or_path), revision=revision))
        except Exception as exc:  # network, authentication or a missing repository
            raise CheckpointFormatError(f"cannot fetch {repo_or_path!r} from the Hub: {exc}") from exc
    return load_folder(path, base_model, **kwargs)
