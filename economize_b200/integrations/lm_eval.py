"""An lm-evaluation-harness model backed by an :class:`~economize_b200.core.model.EfficientModel` (economize
``integrations/lm_eval.py:1-217``).

:class:`EconomizeLM` answers lm-eval's three request types:

* ``generate_until(requests)``: each request's ``args`` are ``(context, gen_kwargs)``; the context is encoded,
  decoded through the model's speculative engine (greedy; ``max_gen_toks`` new tokens at most), and the text is cut
  at the first of ``gen_kwargs["until"]``.
* ``loglikelihood(requests)``: ``(context, continuation)``; one causal pass over both returns the continuation's summed
  log-probability and whether every continuation token is the argmax (lm-eval's ``is_greedy``).
* ``loglikelihood_rolling(requests)``: ``(text,)``; the summed log-probability of the whole text in windows of
  ``max_length`` tokens, each window conditioned on the tail of the previous one.

Scoring passes run the target with every weight transform (quantization, pruning) applied; decoding runs the
configured drafter and verifier. With lm-eval installed, :func:`register` adds the model under ``"economize_b200"``;
the class itself needs only a tokenizer with ``encode`` and ``decode``.
"""

from __future__ import annotations

from typing import Any

import torch

__all__ = ["EconomizeLM", "register"]


def _args(request: Any) -> tuple:
    return tuple(request.args) if hasattr(request, "args") else tuple(request)


class EconomizeLM:
    """lm-eval's model interface over ``model`` and ``tokenizer`` (``decoding``: the DecodeConfig of generations)."""

    def __init__(self, model, tokenizer, *, decoding=None, max_length: int = 4096, max_gen_toks: int = 256,
                 add_bos: bool = False) -> None:
        self.model = model
        self.tokenizer = tokenizer
        self.decoding = decoding
        self.max_length = int(max_length)
        self.max_gen_toks = int(max_gen_toks)
        self.add_bos = add_bos

    @property
    def device(self) -> torch.device:
        return self.model.model.device

    def _encode(self, text: str) -> list[int]:
        try:
            ids = self.tokenizer.encode(text, add_special_tokens=False)
        except TypeError:
            ids = self.tokenizer.encode(text)
        return list(ids)

    def _bos(self) -> list[int]:
        bos = getattr(self.tokenizer, "bos_token_id", None)
        return [bos] if self.add_bos and bos is not None else []

    @torch.no_grad()
    def _scores(self, ids: list[int], start: int) -> tuple[float, bool]:
        """Summed log-probability of ``ids[start:]`` given ``ids[:start]`` and whether each is the argmax."""
        x = torch.tensor(ids, dtype=torch.long, device=self.device)
        logp = torch.log_softmax(self.model(x[None])[0].float(), -1)
        target = x[start:]
        picked = logp[start - 1:-1].gather(1, target[:, None])[:, 0]
        greedy = bool((logp[start - 1:-1].argmax(-1) == target).all())
        return float(picked.sum()), greedy

    def loglikelihood(self, requests) -> list[tuple[float, bool]]:
        out = []
        for r in requests:
            context, continuation = _args(r)[:2]
            ctx = self._bos() + self._encode(context)
            cont = self._encode(continuation)
            if not ctx:  # an empty context: condition on the first continuation token
                ctx, cont = cont[:1], cont[1:]
            ids = (ctx + cont)[-self.max_length:]
            start = max(1, len(ids) - len(cont))
            out.append(self._scores(ids, start) if cont else (0.0, True))
        return out

    def loglikelihood_rolling(self, requests) -> list[float]:
        out = []
        for r in requests:
            (text,) = _args(r)[:1]
            ids = self._bos() + self._encode(text)
            total, pos = 0.0, 1
            while pos < len(ids):
                end = min(len(ids), pos + self.max_length - 1)
                lo = max(0, end - self.max_length)
                window = ids[lo:end]
                total += self._scores(window, pos - lo)[0]
                pos = end
            out.append(total)
        return out

    def generate_until(self, requests) -> list[str]:
        out = []
        for r in requests:
            context, kwargs = _args(r)[:2]
            kwargs = dict(kwargs or {})
            until = kwargs.get("until") or []
            until = [until] if isinstance(until, str) else list(until)
            max_new = int(kwargs.get("max_gen_toks", self.max_gen_toks))
            ids = (self._bos() + self._encode(context))[-(self.max_length - max_new):]
            prompt = torch.tensor(ids, dtype=torch.long, device=self.device)
            tokens = self.model.decode(prompt, max_new, decoding=self.decoding).tokens
            text = self.tokenizer.decode(tokens.tolist())
            cut = min((text.find(s) for s in until if s and s in text), default=-1)
            out.append(text[:cut] if cut >= 0 else text)
        return out


def register() -> type:
    """Register :class:`EconomizeLM` with lm-eval (under ``"economize_b200"``) when lm-eval is installed."""
    from lm_eval.api.model import LM
    from lm_eval.api.registry import register_model

    cls = type("EconomizeHarnessLM", (EconomizeLM, LM), {})
    register_model("economize_b200")(cls)
    return cls
