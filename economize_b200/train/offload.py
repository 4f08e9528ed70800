"""AdamW with its state on the host (economize ``train/offload.py``): the float32 master copy of the trained
parameters and both moments live in pinned CPU memory, so a drafter whose optimizer state would not fit beside the
frozen target trains with only its bf16/fp32 working parameters and gradients on the device.

Every step copies the gradients to the host (non-blocking, one stream synchronization), runs ``torch.optim.AdamW``
on the host tensors, and copies the updated master values back into the device parameters. The update is the one
AdamW computes on the device, up to the host's float32 arithmetic.
"""

from __future__ import annotations

import torch

__all__ = ["OffloadedAdamW"]


class OffloadedAdamW(torch.optim.Optimizer):
    """``torch.optim.AdamW`` over host copies of ``params`` (same hyperparameters); ``param_groups`` expose the
    learning rate to schedulers as usual."""

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.01) -> None:
        params = [p for p in params]
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        pin = torch.cuda.is_available()
        self._host = [p.detach().to("cpu", torch.float32).clone() for p in params]
        if pin:
            self._host = [h.pin_memory() for h in self._host]
        for h in self._host:
            h.requires_grad_(True)
        self._inner = torch.optim.AdamW(self._host, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        self._pairs = list(zip(params, self._host))

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        group = self.param_groups[0]
        for g in self._inner.param_groups:  # a scheduler changes this optimizer's lr: pass it on
            g["lr"] = group["lr"]
        for p, h in self._pairs:
            h.grad = None if p.grad is None else p.grad.detach().to("cpu", torch.float32, non_blocking=True)
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        self._inner.step()
        for p, h in self._pairs:
            p.copy_(h.to(p.device, p.dtype, non_blocking=True))
        return loss

    def zero_grad(self, set_to_none: bool = True) -> None:
        super().zero_grad(set_to_none)
        self._inner.zero_grad(set_to_none)

    def state_dict(self):
        return {"inner": self._inner.state_dict(), "host": [h.detach().clone() for h in self._host],
                "lr": self.param_groups[0]["lr"]}

    def load_state_dict(self, state) -> None:
        self._inner.load_state_dict(state["inner"])
        with torch.no_grad():
            for h, saved in zip(self._host, state["host"]):
                h.copy_(saved)
        self.param_groups[0]["lr"] = state["lr"]
