"""Llama-architecture decoder (Llama-3 8B / 70B shapes) on the sm_100a kernels.

Weights are random (normal, std 1/sqrt(fan_in)) and created directly on the
device, sharded for tensor parallelism: column-parallel QKV and gate/up
(each rank owns whole heads / whole FFN columns), row-parallel o_proj and
down_proj (their partial sums are reduced across ranks by the fused
GEMM + all-reduce kernels of ``parallel.tp``), vocabulary-parallel LM head.

One forward handles a mixed batch: the first ``n_decode`` token rows are
decode tokens (one per running request), the rest are prefill chunks. All
projections, norms and RoPE run once over all rows; attention splits into
the decode kernel (rows [0, n_decode)) and the prefill kernel (the rest).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass, field

import torch

from .. import ops
from .config import ModelConfig

GATE_UP_BLOCK = 64  # gate/up interleave granularity of the SwiGLU GEMM epilogue


def rope_table(cfg: ModelConfig, max_pos: int, device) -> torch.Tensor:
    """[max_pos, head_dim/2, 2] float32 (cos, sin) for rotate-half RoPE."""
    half = cfg.head_dim // 2
    inv = cfg.rope_theta ** (-torch.arange(0, half, dtype=torch.float64) * 2.0 / cfg.head_dim)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.stack([ang.cos(), ang.sin()], dim=-1).to(torch.float32).to(device).contiguous()


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, block: int = GATE_UP_BLOCK) -> torch.Tensor:
    """[I, H] gate and up -> [2I, H] with blocks (gate[j:j+64], up[j:j+64])."""
    I, H = gate.shape
    assert I % block == 0
    g = gate.reshape(I // block, block, H)
    u = up.reshape(I // block, block, H)
    return torch.stack([g, u], dim=1).reshape(2 * I, H).contiguous()


def deinterleave_gate_up(w: torch.Tensor, block: int = GATE_UP_BLOCK):
    I2, H = w.shape
    v = w.reshape(I2 // (2 * block), 2, block, H)
    return v[:, 0].reshape(-1, H), v[:, 1].reshape(-1, H)


@dataclass
class LayerWeights:
    ln_in: torch.Tensor
    qkv: torch.Tensor      # [(hq + 2 hkv) * D, H]   (this rank's heads)
    o: torch.Tensor        # [H, hq * D]
    ln_post: torch.Tensor
    gate_up: torch.Tensor  # [2 * I_local, H] interleaved (dense layers)
    down: torch.Tensor     # [H, I_local]
    moe: object = None     # parallel.ep.MoEWeights for expert layers


@dataclass
class ModelWeights:
    embed: torch.Tensor     # [V, H] (replicated)
    layers: list
    ln_final: torch.Tensor
    lm_head: torch.Tensor   # [V_local, H]
    vocab_offset: int = 0


def _normal(shape, std, device, gen):
    t = torch.empty(shape, dtype=torch.bfloat16, device=device)
    t.normal_(0.0, std, generator=gen)
    return t


def init_weights(cfg: ModelConfig, device, tp_rank: int = 0, tp_size: int = 1, seed: int = 0,
                 moe_builder=None) -> ModelWeights:
    """Random weights of this rank's shard (no full tensor is materialised)."""
    assert cfg.n_q_heads % tp_size == 0 and cfg.n_kv_heads % tp_size == 0
    assert cfg.ffn % (tp_size * GATE_UP_BLOCK) == 0 and cfg.vocab % tp_size == 0 or True
    gen = torch.Generator(device=device)
    gen.manual_seed(seed * 1000003 + tp_rank)
    H, D = cfg.hidden, cfg.head_dim
    hq, hkv = cfg.n_q_heads // tp_size, cfg.n_kv_heads // tp_size
    I = cfg.ffn // tp_size
    ones = lambda: torch.ones(H, dtype=torch.bfloat16, device=device)
    layers = []
    for li in range(cfg.n_layers):
        lw = LayerWeights(
            ln_in=ones(),
            qkv=_normal(((hq + 2 * hkv) * D, H), 1.0 / math.sqrt(H), device, gen),
            o=_normal((H, hq * D), 1.0 / math.sqrt(cfg.n_q_heads * D), device, gen),
            ln_post=ones(),
            gate_up=None if cfg.n_experts else _normal((2 * I, H), 1.0 / math.sqrt(H), device, gen),
            down=None if cfg.n_experts else _normal((H, I), 1.0 / math.sqrt(cfg.ffn), device, gen),
        )
        if cfg.n_experts:
            lw.moe = moe_builder(li, gen)
        layers.append(lw)
    v_local = (cfg.vocab + tp_size - 1) // tp_size
    v_local = (v_local + 127) // 128 * 128  # GEMM row tiles
    # the embedding is replicated: same seed on every rank
    egen = torch.Generator(device=device)
    egen.manual_seed(seed * 1000003 + 7777)
    embed = _normal((cfg.vocab, H), 1.0, device, egen)
    lm = _normal((v_local, H), 1.0 / math.sqrt(H), device, gen)
    return ModelWeights(embed=embed, layers=layers, ln_final=ones(), lm_head=lm,
                        vocab_offset=tp_rank * v_local)


def full_weights(cfg: ModelConfig, seed: int = 0) -> ModelWeights:
    """Unsharded random weights on the CPU (fp32 generator, bf16 storage), for
    comparing tensor-parallel shards against a single-GPU model."""
    g = torch.Generator().manual_seed(seed)
    H, D = cfg.hidden, cfg.head_dim
    rnd = lambda shape, std: (torch.randn(shape, generator=g) * std).to(torch.bfloat16)
    layers = []
    for _ in range(cfg.n_layers):
        layers.append(LayerWeights(
            ln_in=torch.ones(H, dtype=torch.bfloat16),
            qkv=rnd((cfg.qkv_dim, H), 1.0 / math.sqrt(H)),
            o=rnd((H, cfg.n_q_heads * D), 1.0 / math.sqrt(cfg.n_q_heads * D)),
            ln_post=torch.ones(H, dtype=torch.bfloat16),
            gate_up=rnd((2 * cfg.ffn, H), 1.0 / math.sqrt(H)),
            down=rnd((H, cfg.ffn), 1.0 / math.sqrt(cfg.ffn))))
    v = (cfg.vocab + 127) // 128 * 128
    return ModelWeights(embed=rnd((cfg.vocab, H), 1.0), layers=layers,
                        ln_final=torch.ones(H, dtype=torch.bfloat16), lm_head=rnd((v, H), 1.0 / math.sqrt(H)))


def shard_weights(cfg: ModelConfig, full: ModelWeights, rank: int, world: int, device) -> ModelWeights:
    """This rank's tensor-parallel shard of ``full``: whole q/kv heads and
    whole 64-row gate/up blocks per rank, the matching K-slices of o/down,
    and a contiguous vocabulary slice of the LM head."""
    D = cfg.head_dim
    hq, hkv = cfg.n_q_heads // world, cfg.n_kv_heads // world
    I = cfg.ffn // world
    to = lambda t: t.to(device).contiguous()
    layers = []
    for lw in full.layers:
        q = lw.qkv[: cfg.n_q_heads * D].view(cfg.n_q_heads, D, -1)
        k = lw.qkv[cfg.n_q_heads * D:(cfg.n_q_heads + cfg.n_kv_heads) * D].view(cfg.n_kv_heads, D, -1)
        v = lw.qkv[(cfg.n_q_heads + cfg.n_kv_heads) * D:].view(cfg.n_kv_heads, D, -1)
        qkv = torch.cat([q[rank * hq:(rank + 1) * hq].reshape(-1, cfg.hidden),
                         k[rank * hkv:(rank + 1) * hkv].reshape(-1, cfg.hidden),
                         v[rank * hkv:(rank + 1) * hkv].reshape(-1, cfg.hidden)])
        gate, up = deinterleave_gate_up(lw.gate_up)
        gu = interleave_gate_up(gate[rank * I:(rank + 1) * I], up[rank * I:(rank + 1) * I])
        layers.append(LayerWeights(
            ln_in=to(lw.ln_in), qkv=to(qkv), o=to(lw.o[:, rank * hq * D:(rank + 1) * hq * D]),
            ln_post=to(lw.ln_post), gate_up=to(gu), down=to(lw.down[:, rank * I:(rank + 1) * I])))
    v_local = (cfg.vocab + world - 1) // world
    v_local = (v_local + 127) // 128 * 128
    lm = torch.zeros(v_local, cfg.hidden, dtype=torch.bfloat16)
    rows = full.lm_head[rank * v_local:min((rank + 1) * v_local, full.lm_head.shape[0])]
    lm[: rows.shape[0]] = rows
    return ModelWeights(embed=to(full.embed), layers=layers, ln_final=to(full.ln_final), lm_head=to(lm),
                        vocab_offset=rank * v_local)


# residual add + RMSNorm inside the row-parallel projections (1) or as the
# separate add_rmsnorm kernel (0, the default: measured faster, see
# _row_linear_norm)
FUSED_NORM = os.environ.get("SCHED_FUSED_NORM", "0") == "1"
# SCHED_L2_PREFETCH=1: decode attention prefetches the output projection's
# weights into L2 while it streams the KV cache. Off by default: measured on
# B200 (batch-6 Llama-3-8B steps) it made the decode step slower, 4.30-4.32 vs
# 4.23 ms p50 (the prefetches compete with the KV stream and delay the
# producer's first loads).
L2_PREFETCH = os.environ.get("SCHED_L2_PREFETCH", "0") == "1"


@dataclass
class ForwardBatch:
    """Device inputs of one forward (static buffers when graph-captured)."""

    ids: torch.Tensor          # [T] int32
    pos: torch.Tensor          # [T] int32 absolute positions
    slot: torch.Tensor         # [T] int32 KV slot = page * 16 + offset (-1: no write)
    n_tokens: int
    n_decode: int
    block_table: torch.Tensor  # [R, max_pages] int32, rows = batch requests
    kv_lens: torch.Tensor      # [R] int32 (tokens in the cache after this step)
    # decode attention plan
    items: torch.Tensor | None = None       # [n_items, 4] int32
    n_items: int = 0
    part_o: torch.Tensor | None = None
    part_lse: torch.Tensor | None = None
    merge_req: torch.Tensor | None = None
    merge_begin: torch.Tensor | None = None
    n_merge: int = 0
    merge_cnt: torch.Tensor | None = None   # in-kernel merge counters (zero between calls)
    splits: int = 1
    # prefill attention plan
    tiles: torch.Tensor | None = None       # [n_tiles, 4] int32
    n_tiles: int = 0
    # rows whose logits are sampled
    sample_idx: torch.Tensor | None = None  # [S] int64
    n_sample: int = 0
    out_ids: torch.Tensor | None = None     # [S] int32
    # scheduling tables for the woven decode kernel
    slots: dict | None = None
    acquire: int = 0
    grid: int = 0
    # tiered KV: per-layer staging of host-resident pages (engine/tiered_kv.py)
    tier: object = None


class KVCache:
    """Paged KV pool: per layer [pages, Hkv_local, 16, D] for K and for V.

    Zero-initialised: pages beyond a request's last token are read by the
    block-granular decode kernel with probability weight zero, and must hold
    finite values."""

    def __init__(self, cfg: ModelConfig, num_pages: int, device, tp_size: int = 1, page_size: int = 16):
        self.page_size = page_size
        self.num_pages = num_pages
        hkv = cfg.n_kv_heads // tp_size
        self.k = torch.zeros(cfg.n_layers, num_pages, hkv, page_size, cfg.head_dim,
                             dtype=torch.bfloat16, device=device)
        self.v = torch.zeros_like(self.k)

    def bytes(self) -> int:
        return 2 * self.k.numel() * self.k.element_size()


class Llama:
    """Forward pass of one tensor-parallel rank."""

    def __init__(self, cfg: ModelConfig, weights: ModelWeights, kv: KVCache, device,
                 tp=None, max_tokens: int = 8192, max_pos: int = 8192):
        self.cfg = cfg
        self.w = weights
        self.kv = kv
        self.device = torch.device(device)
        self.tp = tp
        self.tp_size = tp.world if tp is not None else 1
        self.hq = cfg.n_q_heads // self.tp_size
        self.hkv = cfg.n_kv_heads // self.tp_size
        self.cos_sin = rope_table(cfg, max_pos, self.device)
        self.sm_scale = 1.0 / math.sqrt(cfg.head_dim)
        self.l2_prefetch = L2_PREFETCH
        self.max_tokens = max_tokens
        # sequence-parallel layer plumbing (tensor-parallel mode "sp"), else None
        self.sp = tp.sequence_parallel(cfg.hidden, max_tokens) if tp is not None else None
        self._sp_out = None
        self._alloc(max_tokens)

    def _alloc(self, T: int) -> None:
        cfg, dev = self.cfg, self.device
        bf = torch.bfloat16
        self.h = torch.empty(T, cfg.hidden, dtype=bf, device=dev)       # residual stream
        self.normed = torch.empty(T, cfg.hidden, dtype=bf, device=dev)
        self.delta = torch.empty(T, cfg.hidden, dtype=bf, device=dev)
        self.qkv = torch.empty(T, (self.hq + 2 * self.hkv) * cfg.head_dim, dtype=bf, device=dev)
        self.q = torch.empty(T, self.hq, cfg.head_dim, dtype=bf, device=dev)
        self.attn = torch.empty(T, self.hq, cfg.head_dim, dtype=bf, device=dev)
        ffn_local = cfg.ffn // self.tp_size
        self.act = torch.empty(T, ffn_local, dtype=bf, device=dev)

    # row-parallel projection: partial sums reduced across TP ranks
    def _row_linear(self, x, w, out):
        if self.tp is None:
            return ops.linear(x, w, out)
        return self.tp.linear_allreduce(x, w, out)

    def _row_linear_norm(self, x, w, out, res, nw, normed) -> None:
        """out = row-parallel x @ w.T, then res += out and normed =
        rmsnorm(res) * nw. By default the separate add_rmsnorm kernel (one
        CTA per row, launched with programmatic dependent launch);
        ``SCHED_FUSED_NORM=1`` does it in the projection kernel itself, where
        the CTA that finishes a token row normalises it, with identical
        results. Measured on one B200 the fused form is slower: the CTA that
        completes the last column tile completes every row of the token tile
        and normalises them one after another (decode step at batch 6: 4.86
        vs 4.37 ms; a 1536-token prefill step: 95 vs 32 ms)."""
        eps = self.cfg.rms_eps
        if not FUSED_NORM:
            self._row_linear(x, w, out)
            ops.add_rmsnorm(out, res, nw, eps, normed)
        elif self.tp is None:
            ops.linear_add_rmsnorm(x, w, out, res, nw, eps, normed)
        else:
            self.tp.linear_allreduce(x, w, out, norm=(res, nw, eps, normed))

    def _attention(self, li: int, b: ForwardBatch) -> None:
        kc, vc = self.kv.k[li], self.kv.v[li]
        nd = b.n_decode
        if nd > 0:
            q = self.q[:nd]
            out = self.attn[:nd]
            stage = b.tier.before_attention(li) if b.tier is not None else None
            ops.attention_decode(q, out, kc, vc, b.block_table, b.items, b.n_items, self.sm_scale,
                                 part_o=b.part_o, part_lse=b.part_lse, merge_cnt=b.merge_cnt,
                                 splits=b.splits, slots=b.slots, woven=b.slots is not None,
                                 acquire=b.acquire, grid=b.grid, stage=stage,
                                 l2_prefetch=self.w.layers[li].o if self.l2_prefetch else None)
            if b.tier is not None:
                b.tier.after_attention(li)
            if b.n_merge > 0 and b.merge_cnt is None:
                ops.attention_merge(b.part_o, b.part_lse, b.merge_req, b.merge_begin, b.n_merge, out)
        if b.n_tiles > 0:
            T = b.n_tokens
            ops.attention_prefill(self.q[nd:T], self.attn[nd:T], kc, vc, b.block_table, b.kv_lens,
                                  b.tiles, b.n_tiles, self.sm_scale)

    def _mlp(self, li: int, x: torch.Tensor, T: int) -> torch.Tensor:
        lw = self.w.layers[li]
        act = ops.linear(x, lw.gate_up, self.act[:T], swiglu=True)
        return self._row_linear(act, lw.down, self.delta[:T])

    def _forward_sp(self, b: ForwardBatch) -> torch.Tensor:
        """Sequence-parallel forward (``parallel/sp.py``): o_proj and down_proj
        reduce-scatter their partial rows to the rank that owns the token,
        which adds the residual and normalises them, then all-gathers the
        normed rows into every rank's copy of the next GEMM's input; that
        GEMM waits per token tile on the rows' ready flags. The residual
        stream ``h`` is only current on the rows this rank owns."""
        cfg, sp = self.cfg, self.sp
        T = b.n_tokens
        h = self.h[:T]
        ops.embedding(b.ids[:T], self.w.embed, h, prev=b.out_ids)
        if b.tier is not None:
            b.tier.begin_forward()
        layers = self.w.layers
        x, ready = self.normed[:T], 0
        ops.add_rmsnorm(h, None, layers[0].ln_in, cfg.rms_eps, x)  # every rank, every row
        for li, lw in enumerate(layers):
            ops.linear_qkv_rope(x, lw.qkv, b.pos[:T], b.slot[:T], self.cos_sin, self.q[:T],
                                self.kv.k[li], self.kv.v[li], self.hq, self.hkv, x_ready=ready)
            self._attention(li, b)
            sp.linear_rs(self.attn[:T].view(T, -1), lw.o)
            x, ready = sp.reduce_norm(h, lw.ln_post, cfg.rms_eps, T)
            act = ops.linear(x, lw.gate_up, self.act[:T], swiglu=True, x_ready=ready)
            sp.linear_rs(act, lw.down)
            nxt = layers[li + 1].ln_in if li + 1 < len(layers) else self.w.ln_final
            x, ready = sp.reduce_norm(h, nxt, cfg.rms_eps, T)
        if b.tier is not None:
            b.tier.end_forward()
        sp.wait_rows(ready, T)  # sampling reads the gathered final rows with library ops
        self._sp_out = x
        return self.sample(b)

    def forward(self, b: ForwardBatch) -> torch.Tensor:
        if self.sp is not None:
            return self._forward_sp(b)
        cfg = self.cfg
        T = b.n_tokens
        h, normed, delta = self.h[:T], self.normed[:T], self.delta[:T]
        ops.embedding(b.ids[:T], self.w.embed, h, prev=b.out_ids)
        if b.tier is not None:
            b.tier.begin_forward()
        layers = self.w.layers
        ops.add_rmsnorm(h, None, layers[0].ln_in, cfg.rms_eps, normed)
        for li, lw in enumerate(layers):
            # normed holds this layer's input norm: from the embedding (layer 0)
            # or from the previous layer's down_proj
            ops.linear_qkv_rope(normed, lw.qkv, b.pos[:T], b.slot[:T], self.cos_sin, self.q[:T],
                                self.kv.k[li], self.kv.v[li], self.hq, self.hkv)
            self._attention(li, b)
            self._row_linear_norm(self.attn[:T].view(T, -1), lw.o, delta, h, lw.ln_post, normed)
            act = ops.linear(normed, lw.gate_up, self.act[:T], swiglu=True)
            nxt = layers[li + 1].ln_in if li + 1 < len(layers) else self.w.ln_final
            self._row_linear_norm(act, lw.down, delta, h, nxt, normed)
        if b.tier is not None:
            b.tier.end_forward()
        return self.sample(b)

    def sample(self, b: ForwardBatch) -> torch.Tensor:
        """Greedy next token of the rows in ``b.sample_idx``."""
        S = b.n_sample
        if S == 0:
            return b.out_ids[:0]
        final = self._sp_out if self.sp is not None else self.normed
        rows = final.index_select(0, b.sample_idx[:S]) if b.sample_idx is not None else final[:S]
        if self.tp is None:
            logits = ops.linear(rows, self.w.lm_head)
            return ops.argmax(logits[:, :self.cfg.vocab], b.out_ids[:S])
        return self.tp.sharded_argmax(rows, self.w.lm_head, self.w.vocab_offset, self.cfg.vocab,
                                      b.out_ids[:S])
