"""Pruning masks.

* magnitude: score ``|W|``.
* Wanda (Sun et al., 2024, "A Simple and Effective Pruning Approach for Large Language Models"): score
  ``|W_ij| * ||X_j||_2`` with the input column norms over calibration tokens, compared within each output row.
* SparseGPT (Frantar & Alistarh, 2023): columns are visited in blocks; within a block the mask removes the entries
  with the smallest ``w^2 / [H^-1]_jj^2`` (per row, or per group of m for N:M) and the removal error of each column is
  propagated to the remaining columns through the upper Cholesky factor of the damped inverse Hessian.
"""

from __future__ import annotations

import torch

__all__ = ["magnitude_scores", "nm_mask", "sparsegpt", "unstructured_mask", "wanda_scores"]


def magnitude_scores(w: torch.Tensor) -> torch.Tensor:
    return w.abs().float()


def wanda_scores(w: torch.Tensor, col_norm: torch.Tensor) -> torch.Tensor:
    return w.abs().float() * col_norm.float()[None, :]


def unstructured_mask(score: torch.Tensor, sparsity: float) -> torch.Tensor:
    """Keep mask removing the ``sparsity`` fraction of lowest scores in every row."""
    n, k = score.shape
    drop = int(k * sparsity)
    mask = torch.ones_like(score, dtype=torch.bool)
    if drop:
        idx = score.topk(drop, -1, largest=False).indices
        mask.scatter_(1, idx, False)
    return mask


def nm_mask(score: torch.Tensor, n: int, m: int) -> torch.Tensor:
    """Keep mask of the ``n`` highest scores in every group of ``m`` consecutive columns."""
    rows, k = score.shape
    g = score.reshape(rows, k // m, m)
    keep = g.topk(n, -1).indices
    return torch.zeros_like(g, dtype=torch.bool).scatter_(-1, keep, True).reshape(rows, k)


@torch.no_grad()
def sparsegpt(weight: torch.Tensor, hessian: torch.Tensor, sparsity: float, nm: tuple[int, int] | None,
              blocksize: int = 128, percdamp: float = 0.01) -> tuple[torch.Tensor, torch.Tensor]:
    """Pruned weights (same dtype) and the keep mask."""
    W = weight.float().clone()
    rows, k = W.shape
    H = hessian.float().clone()
    dead = torch.diag(H) == 0
    H[dead, dead] = 1.0
    W[:, dead] = 0.0
    H += percdamp * torch.mean(torch.diag(H)) * torch.eye(k, device=H.device)
    Hinv = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(H)), upper=True)
    keep = torch.ones_like(W, dtype=torch.bool)
    for i1 in range(0, k, blocksize):
        i2 = min(i1 + blocksize, k)
        W1 = W[:, i1:i2].clone()
        err1 = torch.zeros_like(W1)
        Hinv1 = Hinv[i1:i2, i1:i2]
        d = torch.diag(Hinv1)
        if nm is None:
            score = W1 ** 2 / d[None, :] ** 2
            mask1 = unstructured_mask(score, sparsity)
        else:
            mask1 = torch.ones_like(W1, dtype=torch.bool)
        for i in range(i2 - i1):
            if nm is not None and i % nm[1] == 0:
                blk = W1[:, i:i + nm[1]] ** 2 / d[i:i + nm[1]][None, :] ** 2
                mask1[:, i:i + nm[1]] = nm_mask(blk, nm[0], blk.shape[1]) if blk.shape[1] == nm[1] else True
            w = W1[:, i]
            q = torch.where(mask1[:, i], w, torch.zeros_like(w))
            e = (w - q) / Hinv1[i, i]
            W1[:, i:] -= e[:, None] * Hinv1[i, i:][None, :]
            W1[:, i] = q
            err1[:, i] = e
        W[:, i1:i2] = W1
        keep[:, i1:i2] = mask1
        W[:, i2:] -= err1 @ Hinv[i1:i2, i2:]
    return (W * keep).to(weight.dtype), keep
