"""Thin wrappers: allocate outputs, own the per-device scratch, call the
native launchers on the current stream. No computation happens in Python."""
from __future__ import annotations

import threading

import torch

from .._ext import ext

_lock = threading.Lock()
_status: dict[int, torch.Tensor] = {}
_ws: dict[tuple[int, int], "Workspace"] = {}


def status_buffer(device=None) -> torch.Tensor:
    """The kernels' status words (int32 x 4): [0] a KernelStatus code, set by
    the first bounded wait that gives up or the first out-of-range index
    (0 = OK); for a bad index [1] names the site and [2..3] hold the index."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    with _lock:
        t = _status.get(idx)
        if t is None:
            t = torch.zeros(4, dtype=torch.int32, device=f"cuda:{idx}")
            _status[idx] = t
    return t


STATUS_NAMES = {0: "ok", 1: "tma-timeout", 2: "mma-timeout", 3: "epilogue-timeout",
                4: "peer-timeout", 5: "clc-timeout", 6: "bad-argument", 7: "bad-index"}
INDEX_SITES = {1: "kv page copy: source page", 2: "kv page copy: destination page", 3: "KV append: cache slot",
               4: "embedding: token id", 5: "decode attention: block-table page",
               6: "prefill attention: block-table page"}
# the wait that gave up, for timeouts that record it
WAIT_SITES = {101: "decode producer: task slot free", 102: "decode MMA: task published",
              103: "decode MMA: query rows staged", 104: "decode MMA: task's O buffer free",
              105: "decode softmax: task published"}


class KernelStatusError(RuntimeError):
    def __init__(self, code: int, site: int = 0, index: int = 0):
        self.code, self.site, self.index = code, site, index
        msg = f"kernel reported status {code} ({STATUS_NAMES.get(code, '?')})"
        if code == 7:
            msg += f": {INDEX_SITES.get(site, site)} {index} out of range (access skipped)"
        elif site in WAIT_SITES:
            msg += f" at {WAIT_SITES[site]}"
        super().__init__(msg)


def check_status(device=None, clear: bool = True) -> int:
    """Read (and clear) the status words; raises KernelStatusError on a
    non-zero code."""
    s = status_buffer(device)
    w = s.cpu()
    code = int(w[0])
    if clear and code:
        s.zero_()
    if code:
        site = int(w[1])
        index = int(w[2:4].view(torch.int64)[0]) if code == 7 else 0
        raise KernelStatusError(code, site, index)
    return code


class Workspace:
    """Stream-K scratch of the GEMM: fp32 partial-tile slices and per-tile
    arrival counters. The counters stay zero between calls (the last segment
    of a tile resets its counter), so they are zeroed once here; the slices
    need no clearing (every segment rewrites its own). One workspace per
    stream: calls that share it must be stream-ordered."""

    def __init__(self, device, floats: int = 1 << 24, counters: int = 1 << 16):
        self.device = torch.device(device)
        self.ws = torch.zeros(floats, dtype=torch.float32, device=self.device)
        self.counters = torch.zeros(counters, dtype=torch.int32, device=self.device)

    def ensure(self, floats: int) -> None:
        if floats > self.ws.numel():
            self.ws = torch.zeros(int(floats * 1.25), dtype=torch.float32, device=self.device)


def workspace(device=None, stream_key: int = 0) -> Workspace:
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    with _lock:
        w = _ws.get((idx, stream_key))
        if w is None:
            w = Workspace(f"cuda:{idx}")
            _ws[(idx, stream_key)] = w
    return w


_ws_need: dict[tuple, int] = {}


def _ws_for(x, N, K, grid, ws):
    ws = ws or workspace(x.device)
    key = (x.shape[0], N, K, grid)
    need = _ws_need.get(key)
    if need is None:
        need = int(ext().gemm_ws_floats(x.shape[0], N, K, grid))
        _ws_need[key] = need
    ws.ensure(need)
    return ws


def linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, *,
           swiglu: bool = False, grid: int = 0, ws: Workspace | None = None,
           x_ready: int = 0) -> torch.Tensor:
    """y = x @ w.T on the tcgen05 GEMM. ``swiglu``: w holds interleaved
    gate/up rows (64 gate rows, then their 64 up rows, per 128-row tile) and
    y = silu(gate) * up with N/2 columns. ``grid``: CTAs (0 = one per SM).
    ``x_ready``: device address of per-row ready flags of a gathered x (the
    sequence-parallel all-gather); each token tile is loaded once its rows
    are raised. 0: x is ready."""
    T, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(T, N // 2 if swiglu else N, dtype=torch.bfloat16, device=x.device)
    ws = _ws_for(x, N, K, grid, ws)
    ext().gemm(x, w, out, 1 if swiglu else 0, int(grid), ws.ws, ws.counters, status_buffer(x.device),
               int(x_ready), None, None, None, None, 0.0)
    return out


def linear_add_rmsnorm(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, residual: torch.Tensor,
                       norm_weight: torch.Tensor, eps: float, normed: torch.Tensor, *, grid: int = 0,
                       ws: Workspace | None = None) -> torch.Tensor:
    """out = x @ w.T, then residual += out and normed = rmsnorm(residual) *
    norm_weight in the same kernel: the CTA that writes the last column tile
    of a token row normalises that row, with the arithmetic of
    ``add_rmsnorm`` (bit-identical). Returns normed."""
    T, K = x.shape
    N = w.shape[0]
    ws = _ws_for(x, N, K, grid, ws)
    ext().gemm(x, w, out, 0, int(grid), ws.ws, ws.counters, status_buffer(x.device), 0, residual,
               norm_weight, normed, row_counters(x.device, T), float(eps))
    return normed


_row_cnt: dict[int, torch.Tensor] = {}


def row_counters(device, n: int) -> torch.Tensor:
    """Per-device int32 row counters of the fused norm (zero between calls:
    the kernel that uses a counter resets it). One fixed buffer per device,
    never replaced (CUDA graphs hold its address); calls on one device share
    it, so they must be ordered on one stream."""
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    with _lock:
        t = _row_cnt.get(idx)
        if t is None:
            t = torch.zeros(ROW_COUNTERS, dtype=torch.int32, device=f"cuda:{idx}")
            _row_cnt[idx] = t
    if n > t.numel():
        raise ValueError(f"fused norm over {n} rows: at most {t.numel()} per call")
    return t


ROW_COUNTERS = 16384


def linear_qkv_rope(x, w, pos, slot, cos_sin, q_out, k_cache, v_cache, n_q_heads, n_kv_heads, *,
                    grid: int = 0, ws: Workspace | None = None, x_ready: int = 0):
    """Fused QKV projection + RoPE + KV append: q heads rotated into q_out,
    k heads rotated and v heads copied into their paged-cache slots.
    ``x_ready`` as in ``linear``."""
    ws = _ws_for(x, w.shape[0], x.shape[1], grid, ws)
    ext().gemm_qkv_rope(x, w, pos, slot, cos_sin, q_out, k_cache, v_cache, int(n_q_heads),
                        int(n_kv_heads), int(grid), ws.ws, ws.counters, status_buffer(x.device),
                        int(x_ready))
    return q_out


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor | None, weight: torch.Tensor, eps: float,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """residual += x (in place, when given); returns rmsnorm(residual or x) * weight."""
    if out is None:
        out = torch.empty_like(x)
    ext().add_rmsnorm(x, residual, weight, out, float(eps))
    return out


def rope_kv_append(qkv: torch.Tensor, pos: torch.Tensor, slot: torch.Tensor, cos_sin: torch.Tensor,
                   q_out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                   n_q_heads: int, n_kv_heads: int) -> torch.Tensor:
    ext().rope_kv_append(qkv, pos, slot, cos_sin, q_out, k_cache, v_cache, n_q_heads, n_kv_heads,
                         status_buffer(qkv.device))
    return q_out


def attention_decode(q, out, k_cache, v_cache, block_table, items, num_items, sm_scale, *,
                     part_o=None, part_lse=None, merge_cnt=None, splits=1, slots=None, woven=True,
                     acquire=0, grid=0, pf_blocks=2, dT=1.0, dR=1.0, H=0.25, stage=None,
                     l2_prefetch=None):
    """Paged decode attention. Items (req, kv_begin, kv_end, part) x KV heads
    are the tasks. With ``merge_cnt`` (int32 [requests * Hkv], zero), split
    requests (part = req * splits + s) are merged inside the kernel.
    ``stage=(k, v, split)``: block-table ids >= split index the staging pool
    (k, v) [pages, Hkv, 16, 128] at id - split (tiered KV). ``l2_prefetch``:
    a tensor (the next kernel's weights) whose bytes the CTAs prefetch into
    L2 while they stream the KV cache (a hint: no result depends on it)."""
    s = slots or {}
    pf_ptr = l2_prefetch.data_ptr() if l2_prefetch is not None else 0
    pf_bytes = l2_prefetch.numel() * l2_prefetch.element_size() if l2_prefetch is not None else 0
    sk, sv, split = stage if stage is not None else (None, None, 0)
    ext().attn_decode(q, out, k_cache, v_cache, block_table, items, int(num_items), float(sm_scale),
                      part_o, part_lse, merge_cnt, int(splits), s.get("order"), s.get("ctrl"), s.get("timer"),
                      s.get("queue"), int(s.get("max_tasks", 0)), int(bool(woven)), int(acquire),
                      int(grid), int(pf_blocks), float(dT), float(dR), float(H), sk, sv, int(split),
                      status_buffer(q.device), int(pf_ptr), int(pf_bytes))
    return out


def attention_merge(part_o, part_lse, merge_req, merge_begin, rows, out):
    ext().attn_merge(part_o, part_lse, merge_req, merge_begin, int(rows), out)
    return out


PREFILL_TILE_ROWS = 128  # query rows per prefill-attention tile (the tcgen05 MMA's M)


def attention_prefill(q, out, k_cache, v_cache, block_table, kv_lens, tiles, num_tiles, sm_scale):
    """Causal attention of prefill rows over the paged cache. ``tiles`` [n, 4]
    int32 rows (block-table row, first q row, rows <= PREFILL_TILE_ROWS,
    position of the first row), launched in the given order; rows = 0 marks an
    empty (padding) tile."""
    ext().attn_prefill(q, out, k_cache, v_cache, block_table, kv_lens, tiles, int(num_tiles),
                       float(sm_scale), status_buffer(q.device))
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None,
              prev: torch.Tensor | None = None) -> torch.Tensor:
    """Rows of ``table`` for ``ids``. With ``prev`` (int32 on the device), an
    id -(1 + j) stands for the token ``prev[j]``: a token sampled by the
    previous step that the host has not read yet."""
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
    ext().embedding(ids, table, out, status_buffer(ids.device), prev)
    return out


def argmax(logits: torch.Tensor, out: torch.Tensor | None = None, maxv: torch.Tensor | None = None,
           id_offset: int = 0) -> torch.Tensor:
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    ext().argmax(logits, out, maxv, int(id_offset))
    return out
