"""Expert parallelism (Mixtral-style MoE) over NVLink.

Each rank owns E / world experts, stored as fp8 e4m3 with one fp32 scale
per 128x128 block. A MoE layer on a rank is five kernels (csrc/kernels/moe.cu):
router (top-k softmax) -> dispatch (quantise each assigned token row to fp8
and store it into its expert owner's receive slab over NVLink) -> gate/up
expert GEMM (tcgen05 fp8, waits for every source, SwiGLU) -> activation
quantisation -> down expert GEMM whose epilogue stores each weighted row
back into its source rank's combine buffer -> combine + residual + RMSNorm
on the source. No collective library is involved.

``moe_expert_cap`` is the capacity lever as a plain tensor function (the
reference's python/sched_moe_hook.py:21-65 API); inside the fused path the
same cap is the ``capacity`` of each expert's receive slab.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch

from .. import ops
from .._ext import ext

QB = 128
TN = 64


def quantize_blockwise_fp8(w: torch.Tensor, block: int = QB):
    """[N, K] -> (e4m3 [N, K], fp32 scales [N/block, K/block]); scale = amax / 448."""
    N, K = w.shape
    wb = w.float().reshape(N // block, block, K // block, block)
    amax = wb.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    scale = amax / 448.0
    q = (wb / scale[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    return q.reshape(N, K), scale.contiguous()


def dequantize_blockwise_fp8(q: torch.Tensor, scale: torch.Tensor, block: int = QB) -> torch.Tensor:
    N, K = q.shape
    return (q.float().reshape(N // block, block, K // block, block) * scale[:, None, :, None]).reshape(N, K)


@dataclass
class MoEWeights:
    router: torch.Tensor  # [E, H] bf16 (replicated)
    w13: torch.Tensor     # [E_local * 2I, H] e4m3, gate/up interleaved per 64 rows
    s13: torch.Tensor     # [E_local, 2I/128, H/128] fp32
    w2: torch.Tensor      # [E_local * H, I] e4m3
    s2: torch.Tensor      # [E_local, H/128, I/128] fp32


def build_moe_weights(cfg, rank: int, world: int, gen, device, layer: int = 0) -> MoEWeights:
    """Random expert weights of this rank's experts, quantised per 128x128 block."""
    from ..models.llama import interleave_gate_up
    H, I, E = cfg.hidden, cfg.ffn, cfg.n_experts
    E_local = E // world
    rg = torch.Generator(device=device)
    rg.manual_seed(991 + layer)  # the router is replicated: same on every rank
    router = (torch.randn(E, H, device=device, generator=rg) / math.sqrt(H)).to(torch.bfloat16)
    w13s, s13s, w2s, s2s = [], [], [], []
    for e in range(E_local):
        gate = torch.randn(I, H, device=device, generator=gen) / math.sqrt(H)
        up = torch.randn(I, H, device=device, generator=gen) / math.sqrt(H)
        down = torch.randn(H, I, device=device, generator=gen) / math.sqrt(I)
        q13, s13 = quantize_blockwise_fp8(interleave_gate_up(gate, up))
        q2, s2 = quantize_blockwise_fp8(down)
        w13s.append(q13)
        s13s.append(s13)
        w2s.append(q2)
        s2s.append(s2)
    return MoEWeights(router=router, w13=torch.cat(w13s).contiguous(), s13=torch.stack(s13s).contiguous(),
                      w2=torch.cat(w2s).contiguous(), s2=torch.stack(s2s).contiguous())


def moe_expert_cap(topk_ids, topk_weights, num_experts, capacity_factor=1.25, count=True, min_capacity=8):
    """GShard/Switch expert capacity on routing tensors: each expert keeps at
    most C = capacity_factor * tokens * k / E assignments (in token order);
    the overflow's routing weight becomes 0. Skipped (no-op) when
    C < min_capacity, where per-batch capacity is noise rather than
    imbalance. Fixed shapes, no host sync unless ``count`` (the number of
    dropped assignments is then returned). Returns (weights', dropped)."""
    nt, k = topk_ids.shape
    C = int(capacity_factor * (nt * k) / num_experts)
    if C < min_capacity:
        return topk_weights, (0 if count else None)
    flat_e = topk_ids.reshape(-1).long()
    order = torch.argsort(flat_e, stable=True)
    counts = torch.zeros(num_experts, dtype=torch.long, device=topk_ids.device)
    counts.scatter_add_(0, flat_e, torch.ones_like(flat_e))
    start = torch.cumsum(counts, 0) - counts
    rank_in_expert = torch.arange(flat_e.numel(), device=topk_ids.device) - start[flat_e[order]]
    overflow = torch.zeros(flat_e.numel(), dtype=torch.bool, device=topk_ids.device)
    overflow[order] = rank_in_expert >= C
    w = topk_weights.reshape(-1).masked_fill(overflow, 0.0).reshape(nt, k)
    return w, (int(overflow.sum()) if count else None)


class _LocalBuffer:
    """Single-rank stand-in for a SymmetricBuffer (no torch.distributed)."""

    def __init__(self, nbytes: int):
        self.local, _ = ext().symm_alloc(int(nbytes))
        self.ptrs = [self.local]
        self.world, self.rank = 1, 0

    def close(self):
        if self.local:
            ext().symm_free(self.local)
            self.local = 0


class ExpertParallel:
    """Receive slabs, counters and combine buffers of one MoE layer stack, in
    two sets that alternate between consecutive layer calls.

    A source waits for the owners it routed rows to (their combine rows),
    not for the others: a source that routed nothing to an owner can finish
    layer l and dispatch layer l+1 while that owner is still in layer l,
    whose consumer resets (row counters and done count, cleared at the end of
    the gate/up GEMM) would clear the early arrivals with one set of
    buffers. No source gets two calls ahead: its own gate/up GEMM of layer
    l+1 waits for every source's layer-(l+1) dispatch, which each source
    issues after finishing layer l. So two sets are enough
    (``parallel/ep_protocol.py`` shows one set failing and two passing on
    the CPU). Under CUDA graphs the sets alternate in capture order; every
    step runs every layer, an even number of calls for the named models.
    """

    def __init__(self, cfg, device, group=None, max_tokens: int = 32, capacity: int | None = None):
        import torch.distributed as dist
        self.cfg = cfg
        self.device = torch.device(device)
        distributed = group is not None or (dist.is_available() and dist.is_initialized())
        self.world = dist.get_world_size(group) if distributed else 1
        self.rank = dist.get_rank(group) if distributed else 0
        self.group = group
        E, H, I, K = cfg.n_experts, cfg.hidden, cfg.ffn, cfg.top_k
        assert E % self.world == 0
        self.E, self.E_local, self.H, self.I, self.K = E, E // self.world, H, I, K
        self.max_tokens = max_tokens
        worst = self.world * max_tokens * K  # every token of every rank on one expert
        cap = worst if capacity is None else min(capacity, worst)
        self.capacity = cap
        self.rows = max(TN, (cap + TN - 1) // TN * TN)
        R = self.E_local * self.rows
        # symmetric (peer-visible) region, one allocation carved into parts
        parts = {
            "slab": R * H,                      # fp8
            "slab_scale": R * (H // QB) * 4,     # [H / 128, R]: per K-block rows of token scales
            "slab_meta": R * 4 * 4,
            "counter": max(self.E_local, 4) * 4,
            "done": 16,
            "combine": max_tokens * K * H * 2,  # bf16
            "combine_cnt": 16,
        }
        self.off = {}
        total = 0
        for name, n in parts.items():
            self.off[name] = total
            total += (n + 255) // 256 * 256
        if distributed and self.world > 1:
            from .symm import SymmetricBuffer
            self.bufs = [SymmetricBuffer(total, group) for _ in range(2)]
        else:
            self.bufs = [_LocalBuffer(total) for _ in range(2)]
        self.k = 0
        self.buf = self.bufs[0]
        self.peer = lambda name: [p + self.off[name] for p in self.buf.ptrs]
        self.mine = lambda name: self.buf.ptrs[self.rank] + self.off[name]
        # local scratch
        dev = self.device
        self.act = torch.zeros(R, I, dtype=torch.bfloat16, device=dev)
        self.act_q = torch.zeros(R, I, dtype=torch.uint8, device=dev)
        self.act_scale = torch.zeros(I // QB, R, dtype=torch.float32, device=dev)  # [I / 128, R]
        self.words = torch.zeros(64, dtype=torch.int32, device=dev)  # counters below
        base = self.words.data_ptr()
        self.rows_valid = base            # [E_local] (<= 16)
        self.tiles_done = base + 64
        self.local_done = base + 68
        self.dropped_step = base + 72
        self.dropped_total_ptr = base + 76
        self.arrivals = base + 80
        # stream-K scratch of the expert GEMMs: two fp32 [TN, 128] slices per
        # CTA and one arrival counter per tile (zero between calls)
        self.grid = torch.cuda.get_device_properties(dev).multi_processor_count
        self.ws = torch.empty(self.grid * 2 * TN * 128, dtype=torch.float32, device=dev)
        max_n_tiles = max(2 * I, H) // 128
        self.tile_counters = torch.zeros(self.E_local * max_n_tiles * (self.rows // TN), dtype=torch.int32,
                                         device=dev)
        self.ids = torch.zeros(max_tokens, K, dtype=torch.int32, device=dev)
        self.wts = torch.zeros(max_tokens, K, dtype=torch.float32, device=dev)

    def enable_trace(self, on: bool = True) -> None:
        """Record per-CTA %globaltimer stamps of the two expert GEMMs
        (``self.trace[gemm, cta] = entry, schedule, last TMA, done``)."""
        self.trace = torch.zeros(2, self.grid, 4, dtype=torch.int64, device=self.device) if on else None

    def _trace_ptr(self, i: int) -> int:
        t = getattr(self, "trace", None)
        return t[i].data_ptr() if t is not None else 0

    def dropped_total(self) -> int:
        return int(self.words[19].item())

    def layer(self, w: MoEWeights, x: torch.Tensor, h: torch.Tensor, ln_next: torch.Tensor, y: torch.Tensor,
              eps: float) -> torch.Tensor:
        """x: normalised tokens [T, H]. On return h += MoE(x) and
        y = rmsnorm(h) * ln_next (the next sub-block's input)."""
        E = ext()
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > EP buffers sized for {self.max_tokens}")
        self.buf = self.bufs[self.k]  # this call's buffer set (peer / mine read it)
        self.k ^= 1
        st = ops.status_buffer(x.device)
        ids, wts = self.ids[:T], self.wts[:T]
        if T:
            E.moe_router(x, w.router, ids, wts, self.K)
        E.moe_dispatch(x, ids, wts, T, self.K, self.E, self.E_local, self.rank, self.world, self.capacity,
                       self.rows, self.peer("slab"), self.peer("slab_scale"), self.peer("slab_meta"),
                       self.peer("counter"), self.peer("done"), self.local_done, self.mine("combine"),
                       self.dropped_step, self.dropped_total_ptr, st)
        E.moe_expert_gemm(0, w.w13, self.mine("slab"), self.E_local, 2 * self.I, self.H, self.rows, w.s13,
                          self.mine("slab_scale"), self.act.data_ptr(), self.mine("counter"), self.mine("done"),
                          self.rows_valid, self.tiles_done, self.world, self.capacity, self.mine("slab_meta"),
                          [], [], self.K, self.ws.data_ptr(), self.tile_counters.data_ptr(), self.grid,
                          self._trace_ptr(0), st)
        E.moe_quantize(self.act.data_ptr(), self.act.shape[0], self.I, self.act_q.data_ptr(),
                       self.act_scale.data_ptr(), self.rows_valid, self.rows)
        E.moe_expert_gemm(1, w.w2, self.act_q.data_ptr(), self.E_local, self.H, self.I, self.rows, w.s2,
                          self.act_scale.data_ptr(), 0, self.mine("counter"), self.mine("done"), self.rows_valid,
                          self.tiles_done, self.world, self.capacity, self.mine("slab_meta"),
                          self.peer("combine"), self.peer("combine_cnt"), self.K, self.ws.data_ptr(),
                          self.tile_counters.data_ptr(), self.grid, self._trace_ptr(1), st)
        if T:
            E.moe_combine_norm(self.mine("combine"), self.K, h, ln_next, y, T, eps, self.mine("combine_cnt"),
                               self.dropped_step, self.arrivals, st)
        return y

    def close(self):
        for b in self.bufs:
            b.close()
