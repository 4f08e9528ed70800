"""Run checkpoints: atomic writes, keep-N, resume with optimizer, scheduler, RNG and data position
(economize ``train/checkpoint.py:90-362``). Every checkpoint carries the SHA-256 digests of its files
(``manifest.json``): loading a corrupt one raises, and resuming skips it for the newest intact one."""

from __future__ import annotations

import hashlib
import json
import os
import random
import shutil
import tempfile
from pathlib import Path

import logging

import torch

from ..errors import CheckpointFormatError

__all__ = ["RunCheckpointer", "verify"]

log = logging.getLogger("economize_b200.train")


class RunCheckpointer:
    """Writes ``checkpoint-<step>/`` directories under ``output_dir``; ``final/`` holds the finished run."""

    def __init__(self, output_dir: str | Path, keep: int = 2) -> None:
        self.root = Path(output_dir)
        self.keep = keep
        self.root.mkdir(parents=True, exist_ok=True)

    def _atomic_dir(self, name: str, write) -> Path:
        final = self.root / name
        tmp = Path(tempfile.mkdtemp(prefix=f".{name}.", dir=self.root))
        try:
            write(tmp)
            if final.exists():
                shutil.rmtree(final)
            os.replace(tmp, final)
        except BaseException:
            shutil.rmtree(tmp, ignore_errors=True)
            raise
        return final

    def save(self, step: int, params: dict[str, torch.Tensor], optimizer, scheduler, data_state: dict,
             final: bool = False, result: dict | None = None) -> Path:
        def write(d: Path) -> None:
            torch.save({k: v.detach().cpu() for k, v in params.items()}, d / "weights.pt")
            state = {"step": step, "data": data_state, "torch_rng": torch.get_rng_state(),
                     "python_rng": random.getstate()}
            if torch.cuda.is_available():
                state["cuda_rng"] = torch.cuda.get_rng_state_all()
            if optimizer is not None:
                state["optimizer"] = optimizer.state_dict()
            if scheduler is not None:
                state["scheduler"] = scheduler.state_dict()
            torch.save(state, d / "trainer_state.pt")
            (d / "result.json").write_text(json.dumps(result or {"step": step}))
            manifest = {name: _digest(d / name) for name in ("weights.pt", "trainer_state.pt")}
            (d / "manifest.json").write_text(json.dumps(manifest))

        path = self._atomic_dir("final" if final else f"checkpoint-{step}", write)
        if not final:
            self._prune()
        return path

    def _prune(self) -> None:
        ckpts = sorted(self.checkpoints(), key=lambda p: int(p.name.split("-")[1]))
        for old in ckpts[: max(0, len(ckpts) - self.keep)]:
            shutil.rmtree(old, ignore_errors=True)

    def checkpoints(self) -> list[Path]:
        return [p for p in self.root.glob("checkpoint-*") if p.is_dir() and p.name.split("-")[1].isdigit()]

    def latest(self) -> Path | None:
        """The newest intact checkpoint (a checkpoint whose files no longer match their digests is skipped)."""
        for path in sorted(self.checkpoints(), key=lambda p: int(p.name.split("-")[1]), reverse=True):
            if verify(path):
                return path
            log.warning("skipping corrupt checkpoint %s", path)
        return None

    def finished(self) -> Path | None:
        final = self.root / "final"
        return final if (final / "weights.pt").exists() else None

    @staticmethod
    def load(path: str | Path) -> tuple[dict[str, torch.Tensor], dict]:
        path = Path(path)
        if not verify(path):
            raise CheckpointFormatError(f"checkpoint {path} is corrupt: its files do not match manifest.json")
        weights = torch.load(path / "weights.pt", map_location="cpu", weights_only=True)
        state = torch.load(path / "trainer_state.pt", map_location="cpu", weights_only=False)
        return weights, state


def _digest(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def verify(path: str | Path) -> bool:
    """Whether the checkpoint's files match the SHA-256 digests of its ``manifest.json`` (``True`` without one)."""
    path = Path(path)
    manifest = path / "manifest.json"
    if not manifest.exists():
        return True
    try:
        expected = json.loads(manifest.read_text())
        return all((path / name).exists() and _digest(path / name) == digest for name, digest in expected.items())
    except (OSError, ValueError):
        return False
