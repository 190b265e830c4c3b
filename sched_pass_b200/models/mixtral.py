"""Mixtral-architecture decoder: Llama attention + top-k routed fp8 experts.

Attention is data-parallel across the expert-parallel group (every rank
serves its own requests with replicated attention weights), the experts are
split across ranks (parallel/ep.py). Each layer ends with the fused
combine + residual + RMSNorm, which also produces the next layer's input.
"""
from __future__ import annotations

import torch

from .. import ops
from ..parallel.ep import ExpertParallel, build_moe_weights
from .llama import ForwardBatch, Llama, init_weights


class Mixtral(Llama):
    def __init__(self, cfg, weights, kv, device, ep: ExpertParallel, max_tokens: int = 512, max_pos: int = 8192):
        super().__init__(cfg, weights, kv, device, tp=None, max_tokens=max_tokens, max_pos=max_pos)
        self.ep = ep

    def forward(self, b: ForwardBatch) -> torch.Tensor:
        cfg = self.cfg
        T = b.n_tokens
        h, normed, delta = self.h[:T], self.normed[:T], self.delta[:T]
        layers = self.w.layers
        ops.embedding(b.ids[:T], self.w.embed, h, prev=b.out_ids)
        ops.add_rmsnorm(h, None, layers[0].ln_in, cfg.rms_eps, normed)
        if b.tier is not None:
            b.tier.begin_forward()
        for li, lw in enumerate(layers):
            ops.linear_qkv_rope(normed, lw.qkv, b.pos[:T], b.slot[:T], self.cos_sin, self.q[:T],
                                self.kv.k[li], self.kv.v[li], self.hq, self.hkv)
            self._attention(li, b)
            ops.linear(self.attn[:T].view(T, -1), lw.o, delta)
            ops.add_rmsnorm(delta, h, lw.ln_post, cfg.rms_eps, normed)
            nxt = layers[li + 1].ln_in if li + 1 < len(layers) else self.w.ln_final
            self.ep.layer(lw.moe, normed, h, nxt, normed, cfg.rms_eps)
        if b.tier is not None:
            b.tier.end_forward()
        return self.sample(b)


def mixtral_factory(ep: ExpertParallel, rank: int, world: int):
    """Engine model factory: builds expert weights for this rank and the model."""

    def moe_builder(layer, gen):
        # experts differ across ranks: seed from the shared stream plus the rank
        g = torch.Generator(device=ep.device)
        g.manual_seed(int(torch.randint(0, 2**31 - 1, (1,), generator=gen, device=gen.device).item())
                      * 131 + rank)
        return build_moe_weights(ep.cfg, rank, world, g, ep.device, layer)

    def make(cfg, weights, kv, device, tp, T, max_pos):
        return Mixtral(cfg, weights, kv, device, ep, max_tokens=T, max_pos=max_pos)

    make.moe_builder = moe_builder
    return make
