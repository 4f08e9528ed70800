"""The DFlash block objective (``dflash_block``; economize ``techniques/dflash``): train the draft layer to fill a
whole block in one forward, as it drafts at inference.

For sequences ``tokens [B, S]`` and the frozen target's captured states, every anchor ``a`` gets the block the
drafter builds after it: mask tokens at positions ``a + 1 .. a + m`` (``m = block_size - 1``) with zero features,
attending to the draft layer's entries of the committed context (positions ``<= a``, from the teacher-forced step
that EAGLE-3 training also runs) and bidirectionally to each other. Block slot ``i`` is trained toward the target's
next-token distribution at position ``a + 1 + i`` (KL, the distribution a verified draft must match), the root step
(slot ``-1``, the EAGLE-3 step at ``a``) toward the one at ``a``. Plain PyTorch with autograd; the inference path runs
the same layer on the sm_100a kernels.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ...errors import ConfigError
from ...ops.reference import rmsnorm
from ...runtime.cache import StepBatch
from ...train.objective import OBJECTIVES, Objective, OptimDefaults
from ..eagle3.train import _rope

__all__ = ["DFlashBlockLoss", "block_logits"]


def block_logits(tech, aux: dict[int, torch.Tensor], tokens: torch.Tensor, anchors: torch.Tensor,
                 mask_id: int) -> tuple[torch.Tensor, torch.Tensor]:
    """``(root [B, A, V_d], block [B, A, m, V_d])`` draft logits for ``anchors [A]`` (positions)."""
    layer = tech.layer
    eps = tech.eps
    batch, length = tokens.shape
    heads, kv_heads, hd = layer.heads, layer.kv_heads, layer.head_dim
    group = heads // kv_heads
    m = tech.config.block_size - 1
    n_anchor = anchors.numel()
    cos, sin = layer.rope()
    norm_w, head_w = tech.head_weights()
    sizes = [heads * hd, kv_heads * hd, kv_heads * hd]
    scale = hd ** -0.5

    def mlp_out(residual: torch.Tensor, att: torch.Tensor) -> torch.Tensor:
        a = residual + F.linear(att, layer.wo)
        gate, up = F.linear(rmsnorm(a, layer.post_norm, eps)[0], layer.w_gate_up).chunk(2, -1)
        out = a + F.linear(F.silu(gate) * up, layer.w_down)
        return F.linear(rmsnorm(out, norm_w, eps)[0], head_w).float()

    # ---- the committed context: the teacher-forced step (token p with the features of token p - 1) ----
    g = F.linear(torch.cat([aux[i] for i in tech.aux_layers], -1).to(tech.fc.dtype), tech.fc)
    source = torch.cat([torch.zeros_like(g[:, :1]), g[:, :-1]], 1)
    x_e = rmsnorm(tech.model.embed_tokens(tokens).to(tech.fc.dtype), tech.input_norm, eps)[0]
    x_h = rmsnorm(source, tech.hidden_norm, eps)[0]
    residual = x_h if tech.config.norm_before_residual else source
    q, k, v = F.linear(torch.cat([x_e, x_h], -1), layer.wqkv, layer.bqkv).split(sizes, -1)
    c, s = cos[:length], sin[:length]
    q = _rope(q.reshape(batch, length, heads, hd).transpose(1, 2), c, s)
    k = _rope(k.reshape(batch, length, kv_heads, hd).transpose(1, 2), c, s).repeat_interleave(group, 1)
    v = v.reshape(batch, length, kv_heads, hd).transpose(1, 2).repeat_interleave(group, 1)
    pos = torch.arange(length, device=tokens.device)
    scores = torch.matmul(q, k.transpose(-1, -2)) * scale
    scores = scores.masked_fill(pos[None, :] > pos[:, None], float("-inf"))
    att = torch.matmul(torch.softmax(scores.float(), -1).to(q.dtype), v)
    ctx = att.transpose(1, 2).reshape(batch, length, heads * hd)
    root = mlp_out(residual[:, anchors], ctx[:, anchors])  # [B, A, V]

    # ---- the blocks: mask tokens with zero features after every anchor ----
    bpos = anchors[:, None] + 1 + torch.arange(m, device=tokens.device)[None]  # [A, m]
    emb = tech.model.embed_tokens(torch.full((1,), mask_id, device=tokens.device)).to(tech.fc.dtype)
    xb_e = rmsnorm(emb, tech.input_norm, eps)[0].expand(n_anchor * m, -1)
    zero = torch.zeros_like(xb_e)
    xb_h = rmsnorm(zero, tech.hidden_norm, eps)[0]
    qb, kb, vb = F.linear(torch.cat([xb_e, xb_h], -1), layer.wqkv, layer.bqkv).split(sizes, -1)
    cb, sb = cos[bpos.reshape(-1)], sin[bpos.reshape(-1)]
    qb = _rope(qb.reshape(1, n_anchor * m, heads, hd).transpose(1, 2), cb, sb)  # [1, H, A*m, D]
    kb = _rope(kb.reshape(1, n_anchor * m, kv_heads, hd).transpose(1, 2), cb, sb).repeat_interleave(group, 1)
    vb = vb.reshape(1, n_anchor * m, kv_heads, hd).transpose(1, 2).repeat_interleave(group, 1)
    qb = qb.reshape(1, heads, n_anchor, m, hd)
    kb = kb.reshape(1, heads, n_anchor, m, hd)
    vb = vb.reshape(1, heads, n_anchor, m, hd)
    s_ctx = torch.einsum("xhamd,bhsd->bhams", qb, k) * scale  # [B, H, A, m, S]
    s_ctx = s_ctx.masked_fill(pos[None, None, None, None, :] > anchors[None, None, :, None, None], float("-inf"))
    s_blk = torch.einsum("xhamd,xhand->xhamn", qb, kb).expand(batch, -1, -1, -1, -1) * scale  # [B, H, A, m, m]
    probs = torch.softmax(torch.cat([s_ctx, s_blk], -1).float(), -1).to(qb.dtype)
    attb = torch.einsum("bhams,bhsd->bhamd", probs[..., :length], v) + \
        torch.einsum("bhamn,xhand->bhamd", probs[..., length:], vb)
    attb = attb.permute(0, 2, 3, 1, 4).reshape(batch, n_anchor, m, heads * hd)
    # the block's sources are zero, so its residual is zero whether or not it is normed first
    block = mlp_out(torch.zeros(batch, n_anchor, m, tech.model.config.hidden_size, dtype=attb.dtype,
                                device=attb.device), attb)
    return root, block


@OBJECTIVES.register("dflash_block")
class DFlashBlockLoss(Objective):
    """KL from the frozen target's next-token distributions to the DFlash root and block drafts (module docstring);
    ``anchors``: anchor positions sampled per batch."""

    name = "dflash_block"
    defaults = OptimDefaults(lr=1e-3, warmup_steps=10)

    def __init__(self, model, anchors: int = 16) -> None:
        super().__init__(model)
        tech = model.techniques["dflash"] if "dflash" in model.techniques.keys() else None
        if tech is None:
            raise ConfigError("dflash_block trains an attached dflash technique")
        self.tech = tech
        self.anchors = anchors
        v = tech.model.config.vocab_size
        self.mask_id = tech.config.mask_token_id if tech.config.mask_token_id is not None else v - 1

    def parameters(self):
        return [p for p in self.tech.parameters() if p.requires_grad]

    def loss(self, tokens: torch.Tensor):
        tech = self.tech
        model = tech.model
        b, s = tokens.shape
        m = tech.config.block_size - 1
        if s < m + 3:
            raise ConfigError(f"dflash_block needs sequences of at least block_size + 2 = {m + 3} tokens")
        with torch.no_grad():
            cache = model.new_cache(b, ((s + 127) // 128) * 128)
            lengths = torch.full((b,), s, dtype=torch.int32, device=tokens.device)
            hidden, aux = model.forward_step(tokens, StepBatch.prefill(lengths, s), cache, capture=tech.aux_layers)
            teacher = torch.log_softmax(model.logits(hidden).float(), -1)  # [B, S, V]: predicts p + 1
        g = torch.Generator().manual_seed(int(tokens.sum()) & 0x7FFFFFFF)
        top = s - m - 1  # anchors a with a + 1 + (m - 1) <= s - 1
        anchors = torch.randperm(top, generator=g)[: self.anchors].sort().values.to(tokens.device)
        root, block = block_logits(tech, aux, tokens, anchors, self.mask_id)
        d2t = tech.d2t
        ids = torch.arange(tech.draft_vocab, device=tokens.device)
        target_ids = ids + d2t[ids]

        def kl(logits: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
            t = teacher[:, pos][..., target_ids]
            t = t - torch.logsumexp(t, -1, keepdim=True)  # the target's distribution on the draft vocabulary
            return F.kl_div(torch.log_softmax(logits, -1), t, log_target=True, reduction="batchmean")

        loss_root = kl(root, anchors)
        bpos = anchors[:, None] + 1 + torch.arange(m, device=tokens.device)[None]
        loss_block = kl(block.reshape(b, -1, block.shape[-1]), bpos.reshape(-1))
        loss = loss_root + loss_block
        with torch.no_grad():
            acc = (block.argmax(-1) == teacher[:, bpos][..., target_ids].argmax(-1)).float().mean()
        return loss, {"loss": float(loss.detach()), "root_kl": float(loss_root.detach()),
                      "block_kl": float(loss_block.detach()), "block_acc": float(acc)}
