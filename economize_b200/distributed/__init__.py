"""Multi-process execution (``economize.distributed`` in the reference): process-group set-up, tensor-parallel
loading of a model, and the drafter-on-another-device speculative decoder (``economize_b200.distributed.ssd``)."""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist

from ..parallel.tp import TPGroup, shard_model, tp_argmax

__all__ = ["TPGroup", "init_distributed", "load_tensor_parallel", "shard_model", "tensor_parallel", "tp_argmax"]


def init_distributed(backend: str | None = None, timeout_s: float = 300.0) -> TPGroup:
    """Initialise ``torch.distributed`` from the ``torchrun`` environment (NCCL on GPUs, Gloo on CPUs) and return
    the tensor-parallel group of all ranks (the current device is ``LOCAL_RANK``)."""
    if not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        kwargs = {}
        if backend == "nccl":
            local = int(os.environ.get("LOCAL_RANK", "0"))
            torch.cuda.set_device(local)
            kwargs["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kwargs)
    return TPGroup(dist.get_rank(), dist.get_world_size(), None)


def tensor_parallel(model, tp: TPGroup | None = None, fused: bool = False, max_rows: int = 4096):
    """Shard an engine model (or the engine model of an :class:`~economize_b200.EfficientModel`) over ``tp``
    (default: all ranks). With ``fused`` passes of up to ``max_rows`` tokens run sequence-parallel on the fused
    GEMM -> reduce-scatter and all-gather -> GEMM kernels (NVLink peer stores); longer ones take NCCL."""
    from ..core.model import EfficientModel

    target = model.model if isinstance(model, EfficientModel) else model
    tp = tp or TPGroup(dist.get_rank(), dist.get_world_size(), None)
    if fused and tp.size > 1:
        from ..parallel.sp import SequenceParallel

        tp.fused = True
        tp.sp = SequenceParallel(tp, target.config.hidden_size, max_rows=max_rows)
    shard_model(target, tp)
    if isinstance(model, EfficientModel):
        model.refresh()
    return model


def load_tensor_parallel(name_or_model, *, dtype: torch.dtype = torch.bfloat16, fused: bool = False, **kwargs):
    """Load a Hugging Face causal LM (an id, a path or a module) into the engine and shard it over all ranks of the
    ``torchrun`` job (economize's ``load_tensor_parallel``)."""
    from ..models.llama import CausalLM

    tp = init_distributed()
    if isinstance(name_or_model, str):
        import transformers

        hf = transformers.AutoModelForCausalLM.from_pretrained(name_or_model, dtype=dtype, **kwargs)
    else:
        hf = name_or_model
    device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"
    model = hf if isinstance(hf, CausalLM) else CausalLM.from_hf(hf, dtype=dtype, device=device)
    return tensor_parallel(model, tp, fused=fused)
