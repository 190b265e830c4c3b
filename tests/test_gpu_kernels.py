"""Numerics of the sm_100a kernels against plain fp32 PyTorch statements."""
import math

import numpy as np
import pytest
import torch

from sched_pass_b200 import ops
from sched_pass_b200.models import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _clean_status():
    yield
    ops.check_status()


# ------------------------------------------------------------------ GEMM
@pytest.mark.parametrize("T", [1, 5, 16, 33, 64, 100, 128, 200, 257])
@pytest.mark.parametrize("NK", [(128, 64), (384, 256), (1024, 512), (6144, 4096)])
@pytest.mark.parametrize("grid", [0, 7, 148])
def test_gemm_matches_fp32(T, NK, grid):
    N, K = NK
    g = torch.Generator(device=DEV).manual_seed(T * 31 + N)
    x = torch.randn(T, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV, generator=g) / math.sqrt(K)).to(torch.bfloat16)
    y = ops.linear(x, w, grid=grid)
    torch.cuda.synchronize()
    assert rel_err(y, ref.linear(x, w)) < 1e-2


@pytest.mark.parametrize("T", [3, 64, 300])
@pytest.mark.parametrize("grid", [0, 5])
def test_gemm_swiglu(T, grid):
    I, K = 256, 512
    g = torch.Generator(device=DEV).manual_seed(7)
    x = torch.randn(T, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(2 * I, K, device=DEV, generator=g) / math.sqrt(K)).to(torch.bfloat16)
    y = ops.linear(x, w, swiglu=True, grid=grid)
    torch.cuda.synchronize()
    assert y.shape == (T, I)
    assert rel_err(y, ref.swiglu_linear(x, w)) < 1e-2


def test_gemm_split_workspace_stays_clean():
    # different problems through one workspace: none may see another's partial
    # sums, the arrival counters return to zero, and split-K is deterministic
    x = torch.randn(8, 1024, device=DEV).to(torch.bfloat16)
    w1 = torch.randn(512, 1024, device=DEV).to(torch.bfloat16)
    w2 = torch.randn(512, 1024, device=DEV).to(torch.bfloat16)
    ys = []
    for w in (w1, w2, w1):
        y = ops.linear(x, w, grid=6)
        assert rel_err(y, ref.linear(x, w)) < 1e-2
        ys.append(y)
    assert torch.equal(ys[0], ys[2])
    ws = ops.workspace()
    torch.cuda.synchronize()
    assert ws.counters.abs().max().item() == 0


def test_gemm_large_prefill_shape():
    T, N, K = 1536, 1024, 4096
    x = torch.randn(T, K, device=DEV).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV) / 64).to(torch.bfloat16)
    assert rel_err(ops.linear(x, w), ref.linear(x, w)) < 1e-2


@pytest.mark.parametrize("T", [1, 9, 40, 130])
@pytest.mark.parametrize("grid", [0, 11])
def test_gemm_qkv_rope_kv_append(T, grid):
    from sched_pass_b200.models.config import LLAMA_TINY
    from sched_pass_b200.models.llama import rope_table
    cfg = LLAMA_TINY
    Hq, Hkv, D, H = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, cfg.hidden
    cs = rope_table(cfg, 4096, DEV)
    g = torch.Generator(device=DEV).manual_seed(T)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn((Hq + 2 * Hkv) * D, H, device=DEV, generator=g) / math.sqrt(H)).to(torch.bfloat16)
    pos = torch.randint(0, 4000, (T,), device=DEV, dtype=torch.int32)
    pages = 64
    slot = torch.randperm(pages * 16, device=DEV)[:T].to(torch.int32)
    slot[0] = -1  # a padding row writes no cache entry
    kc = torch.zeros(pages, Hkv, 16, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=DEV)
    ops.linear_qkv_rope(x, w, pos, slot, cs, q, kc, vc, Hq, Hkv, grid=grid)
    torch.cuda.synchronize()
    qkv = ref.linear(x, w).to(torch.bfloat16).view(T, Hq + 2 * Hkv, D)
    assert rel_err(q, ref.rope(qkv[:, :Hq], pos, cs)) < 1e-2
    k_ref = ref.rope(qkv[:, Hq:Hq + Hkv], pos, cs)
    for t in range(T):
        s = int(slot[t])
        if s < 0:
            continue
        assert rel_err(kc[s // 16, :, s % 16], k_ref[t]) < 1e-2
        assert rel_err(vc[s // 16, :, s % 16], qkv[t, Hq + Hkv:]) < 1e-2
    if T > 1:
        assert kc[slot[1:].long() // 16].abs().sum() > 0


@pytest.mark.parametrize("T,N,K,swiglu", [
    (600, 2048, 1024, False), (1030, 4096, 512, True), (256, 512, 256, False), (1536, 1024, 4096, False),
    (1, 512, 512, False),
])
def test_gemm_cta_pair_matches_fp32(T, N, K, swiglu, monkeypatch):
    """The CTA-pair GEMM (tcgen05.mma.cta_group::2, 256 x 256 tiles split over
    a cluster of two CTAs), forced for every eligible shape, against fp32:
    plain store and SwiGLU, token counts that do not fill the last tile."""
    monkeypatch.setenv("SCHED_GEMM_PAIR", "1")
    g = torch.Generator(device=DEV).manual_seed(T + N)
    x = torch.randn(T, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV, generator=g) / math.sqrt(K)).to(torch.bfloat16)
    got = ops.linear(x, w, swiglu=swiglu)
    torch.cuda.synchronize()
    want = ref.swiglu_linear(x, w) if swiglu else ref.linear(x, w)
    assert rel_err(got, want) < 1e-2
    monkeypatch.setenv("SCHED_GEMM_PAIR", "0")
    assert rel_err(ops.linear(x, w, swiglu=swiglu), want) < 1e-2


@pytest.mark.parametrize("T,N,K,swiglu", [
    (1536, 4096, 4096, False), (256, 4096, 14336, False), (512, 4096, 4096, True),
])
def test_gemm_cta_pair_k_ranges(T, N, K, swiglu, monkeypatch):
    """The CTA-pair GEMM with the tiles of its last, partly filled wave split
    into k-ranges (fp32 partials in the workspace; once all have arrived,
    each k-range unit sums a slice of the tile in split order), on the
    automatic plan: against fp32, bit-identical over repeated calls (arrival
    order does not matter), and close to the same kernel with every tile
    whole."""
    from sched_pass_b200._ext import ext
    monkeypatch.delenv("SCHED_GEMM_PAIR", raising=False)
    monkeypatch.delenv("SCHED_GEMM_PAIR_SPLIT", raising=False)
    ws = ops.workspace(DEV)
    np_, whole, splits = ext().gemm_pair_plan(T, N, K, 1 if swiglu else 0, ws.ws.numel(), ws.counters.numel())
    assert np_ > 0 and splits > 1, (np_, whole, splits)
    g = torch.Generator(device=DEV).manual_seed(T + K)
    x = torch.randn(T, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV, generator=g) / math.sqrt(K)).to(torch.bfloat16)
    got = ops.linear(x, w, swiglu=swiglu)
    again = ops.linear(x, w, swiglu=swiglu)
    torch.cuda.synchronize()
    want = ref.swiglu_linear(x, w) if swiglu else ref.linear(x, w)
    assert rel_err(got, want) < 1e-2
    assert torch.equal(got, again)
    monkeypatch.setenv("SCHED_GEMM_PAIR_SPLIT", "0")
    assert ext().gemm_pair_plan(T, N, K, 1 if swiglu else 0, ws.ws.numel(), ws.counters.numel())[2] == 1
    assert rel_err(ops.linear(x, w, swiglu=swiglu), got) < 1e-2


def test_gemm_cta_pair_qkv_rope(monkeypatch):
    """The RoPE + KV-append epilogue on the CTA-pair schedule: rotated
    queries against fp32, and queries, keys and values (written into their
    cache pages) against the single-CTA schedule."""
    from sched_pass_b200.models.config import LLAMA_TINY
    from sched_pass_b200.models.llama import rope_table
    cfg = LLAMA_TINY
    Hq, Hkv, D, H = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, cfg.hidden
    cs = rope_table(cfg, 4096, DEV)
    T = 700
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn((Hq + 2 * Hkv) * D, H, device=DEV, generator=g) / math.sqrt(H)).to(torch.bfloat16)
    pos = torch.randint(0, 4000, (T,), device=DEV, dtype=torch.int32)
    slot = torch.randperm(64 * 16, device=DEV)[:T].to(torch.int32)

    def run(mode):
        monkeypatch.setenv("SCHED_GEMM_PAIR", mode)
        kc = torch.zeros(64, Hkv, 16, D, dtype=torch.bfloat16, device=DEV)
        vc = torch.zeros_like(kc)
        q = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=DEV)
        ops.linear_qkv_rope(x, w, pos, slot, cs, q, kc, vc, Hq, Hkv)
        torch.cuda.synchronize()
        return q, kc, vc
    qp, kp, vp = run("1")
    q1, k1, v1 = run("0")
    qkv = ref.linear(x, w).to(torch.bfloat16).view(T, Hq + 2 * Hkv, D)
    assert rel_err(qp, ref.rope(qkv[:, :Hq], pos, cs)) < 1e-2
    assert rel_err(qp, q1) < 1e-2 and rel_err(kp, k1) < 1e-2 and rel_err(vp, v1) < 1e-2


# ------------------------------------------------------------------ elementwise
def test_add_rmsnorm():
    T, H = 7, 4096
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    r = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    w = torch.randn(H, device=DEV).to(torch.bfloat16)
    r0 = r.clone()
    y = ops.add_rmsnorm(x, r, w, 1e-5)
    s = (x.float() + r0.float()).to(torch.bfloat16)
    assert torch.equal(r, s)
    assert rel_err(y, ref.rmsnorm(s, w, 1e-5)) < 1e-2
    y2 = ops.add_rmsnorm(x, None, w, 1e-5)
    assert rel_err(y2, ref.rmsnorm(x, w, 1e-5)) < 1e-2


def test_rope_kv_append():
    from sched_pass_b200.models.config import LLAMA_TINY
    from sched_pass_b200.models.llama import rope_table
    cfg = LLAMA_TINY
    T, Hq, Hkv, D = 5, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    cs = rope_table(cfg, 1024, DEV)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=DEV).to(torch.bfloat16)
    pos = torch.tensor([0, 3, 17, 100, 999], dtype=torch.int32, device=DEV)
    slot = torch.tensor([5 * 16 + 0, 2 * 16 + 3, 7 * 16 + 1, -1, 0], dtype=torch.int32, device=DEV)
    kc = torch.zeros(8, Hkv, 16, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=DEV)
    ops.rope_kv_append(qkv, pos, slot, cs, q, kc, vc, Hq, Hkv)
    v = qkv.view(T, Hq + 2 * Hkv, D)
    q_ref = ref.rope(v[:, :Hq], pos, cs)
    k_ref = ref.rope(v[:, Hq:Hq + Hkv], pos, cs)
    assert rel_err(q, q_ref) < 1e-2
    for t in range(T):
        s = int(slot[t])
        if s < 0:
            continue
        assert rel_err(kc[s // 16, :, s % 16], k_ref[t]) < 1e-2
        assert torch.equal(vc[s // 16, :, s % 16], v[t, Hq + Hkv:])


def test_embedding_and_argmax():
    table = torch.randn(1000, 512, device=DEV).to(torch.bfloat16)
    ids = torch.tensor([3, 999, 0, 17], dtype=torch.int32, device=DEV)
    assert torch.equal(ops.embedding(ids, table), table[ids.long()])
    logits = torch.randn(6, 128256, device=DEV).to(torch.bfloat16)
    logits[2, 77777] = 100.0
    got = ops.argmax(logits)
    assert torch.equal(got.long(), logits.float().argmax(-1))
    assert got[2].item() == 77777


def test_argmax_rows_of_any_pitch():
    """Rows whose pitch is not a multiple of 8 elements (an odd vocabulary
    shard, a column slice) are read without 16-byte vector loads; the plain
    argmax and the in-kernel (max, id) exchange (one rank) agree with torch."""
    from sched_pass_b200._ext import ext
    for V, cols in ((1007, 1007), (1004, 1003), (2048, 2045)):
        full = torch.randn(6, V, device=DEV).to(torch.bfloat16)
        logits = full[:, :cols]
        want = logits.float().argmax(-1)
        assert torch.equal(ops.argmax(logits).long(), want)
        set_lines = 1024
        buf = torch.zeros(2 * set_lines * 4, dtype=torch.int32, device=DEV)
        state = torch.zeros(2, dtype=torch.int32, device=DEV)
        out = torch.empty(6, dtype=torch.int32, device=DEV)
        for _ in range(3):  # epochs advance across calls
            ext().argmax_exchange(logits, out, 0, [buf.data_ptr()], 0, state, set_lines, ops.status_buffer(DEV))
            torch.cuda.synchronize()
            assert torch.equal(out.long(), want)


def test_launch_error_raises_and_the_process_survives():
    """A launcher that refuses a call (here a GEMM whose N is not a multiple
    of the 128-row tile) raises RuntimeError in Python; the next valid call
    works (the binding records the code, the Python wrapper raises it)."""
    x = torch.randn(3, 512, device=DEV).to(torch.bfloat16)
    with pytest.raises(RuntimeError, match="gemm launch failed"):
        ops.linear(x, torch.randn(1004, 512, device=DEV).to(torch.bfloat16))
    w = torch.randn(1024, 512, device=DEV).to(torch.bfloat16)
    assert rel_err(ops.linear(x, w), x.float() @ w.float().t()) < 1e-2


# ------------------------------------------------------------------ decode attention

def test_embedding_takes_negative_ids_from_the_previous_step():
    """id -(1 + j) with ``prev`` reads token prev[j] (a token the previous
    step sampled that only the device holds yet); other ids read directly."""
    table = torch.randn(1000, 256, device="cuda").to(torch.bfloat16)
    prev = torch.tensor([5, 7, 999], dtype=torch.int32, device="cuda")
    ids = torch.tensor([3, -1, -3, 4, -2], dtype=torch.int32, device="cuda")
    out = ops.embedding(ids, table, prev=prev)
    torch.cuda.synchronize()
    ops.check_status()
    assert torch.equal(out, table[torch.tensor([3, 5, 999, 4, 7], device="cuda")])

def make_paged(B, Hkv, lens, seed=0, pages_extra=7):
    D = 128
    total_pages = sum((int(n) + 15) // 16 for n in lens) + pages_extra
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(total_pages, generator=g)
    kc = torch.randn(total_pages, Hkv, 16, D, generator=g).to(torch.bfloat16).to(DEV)
    vc = torch.randn(total_pages, Hkv, 16, D, generator=g).to(torch.bfloat16).to(DEV)
    maxp = max((int(n) + 15) // 16 for n in lens)
    bt = torch.zeros(B, maxp, dtype=torch.int32)
    k = 0
    for b, n in enumerate(lens):
        npg = (int(n) + 15) // 16
        bt[b, :npg] = perm[k:k + npg]
        k += npg
    return kc, vc, bt.to(DEV)


def run_decode(q, kc, vc, bt, lens, S=1, slots=None, woven=False, acquire=0, grid=0):
    from sched_pass_b200.engine import native
    B, Hq, D = q.shape
    items, mreq, mbeg = native.plan_decode(np.asarray(lens, dtype=np.int32), S)
    it = torch.from_numpy(items).to(DEV)
    out = torch.zeros_like(q)
    po = pl = None
    if S > 1:
        po = torch.zeros(B * S, Hq, D, dtype=torch.float32, device=DEV)
        pl = torch.zeros(B * S, Hq, dtype=torch.float32, device=DEV)
    ops.attention_decode(q, out, kc, vc, bt, it, items.shape[0], 1 / math.sqrt(D), part_o=po,
                         part_lse=pl, slots=slots, woven=woven, acquire=acquire, grid=grid)
    if S > 1:
        ops.attention_merge(po, pl, torch.from_numpy(mreq).to(DEV), torch.from_numpy(mbeg).to(DEV), B, out)
    torch.cuda.synchronize()
    return out, items


LENS = [1, 15, 16, 17, 127, 128, 129, 300, 1000, 2049]


@pytest.mark.parametrize("G", [1, 4, 8])
def test_decode_attention_stock(G):
    Hkv = 2
    B = len(LENS)
    kc, vc, bt = make_paged(B, Hkv, LENS, seed=G)
    q = torch.randn(B, Hkv * G, 128, device=DEV).to(torch.bfloat16)
    out, _ = run_decode(q, kc, vc, bt, LENS)
    r = ref.decode_attention_paged(q, kc, vc, bt, LENS, 1 / math.sqrt(128))
    assert rel_err(out, r) < 2e-2


@pytest.mark.parametrize("S", [2, 3, 8])
def test_decode_attention_split_kv(S):
    Hkv, G = 2, 4
    B = len(LENS)
    kc, vc, bt = make_paged(B, Hkv, LENS, seed=S)
    q = torch.randn(B, Hkv * G, 128, device=DEV).to(torch.bfloat16)
    out, _ = run_decode(q, kc, vc, bt, LENS, S=S)
    r = ref.decode_attention_paged(q, kc, vc, bt, LENS, 1 / math.sqrt(128))
    assert rel_err(out, r) < 2e-2


@pytest.mark.parametrize("S", [2, 5])
@pytest.mark.parametrize("acquire", [0, 2])
def test_decode_in_kernel_merge(S, acquire):
    from sched_pass_b200.engine import native
    Hkv, G = 2, 4
    B = len(LENS)
    kc, vc, bt = make_paged(B, Hkv, LENS, seed=30 + S)
    q = torch.randn(B, Hkv * G, 128, device=DEV).to(torch.bfloat16)
    items, _, _ = native.plan_decode(np.asarray(LENS, dtype=np.int32), S)
    it = torch.from_numpy(items).to(DEV)
    po = torch.zeros(B * S, Hkv * G, 128, dtype=torch.float32, device=DEV)
    pl = torch.zeros(B * S, Hkv * G, dtype=torch.float32, device=DEV)
    cnt = torch.zeros(B * Hkv, dtype=torch.int32, device=DEV)
    p = _plane(items.shape[0] * Hkv)
    if acquire == 2:
        p.set_num_tasks(items.shape[0] * Hkv)
        p.push()
    r = ref.decode_attention_paged(q, kc, vc, bt, LENS, 1 / math.sqrt(128))
    outs = []
    for grid in (0, 37):
        out = torch.zeros_like(q)
        ops.attention_decode(q, out, kc, vc, bt, it, items.shape[0], 1 / math.sqrt(128), part_o=po,
                             part_lse=pl, merge_cnt=cnt, splits=S, slots=p.slots(), woven=True,
                             acquire=acquire, grid=grid if acquire == 0 else 0)
        torch.cuda.synchronize()
        assert rel_err(out, r) < 2e-2
        assert int(cnt.abs().sum()) == 0
        outs.append(out)
    assert torch.equal(outs[0], outs[1])


def _plane(n_tasks):
    from sched_pass_b200.runtime.sched_rt import SchedPlane
    return SchedPlane(max_tasks=max(n_tasks, 64), device=DEV, mode="device")


def test_decode_levers_null_tables_are_bit_exact():
    Hkv, G = 2, 4
    B = len(LENS)
    kc, vc, bt = make_paged(B, Hkv, LENS, seed=11)
    q = torch.randn(B, Hkv * G, 128, device=DEV).to(torch.bfloat16)
    stock, _ = run_decode(q, kc, vc, bt, LENS, woven=False)
    woven_null, _ = run_decode(q, kc, vc, bt, LENS, woven=True, slots=None)
    assert torch.equal(stock, woven_null)
    p = _plane(B * Hkv)
    neutral, _ = run_decode(q, kc, vc, bt, LENS, woven=True, slots=p.slots())
    assert torch.equal(stock, neutral)


def test_decode_pi_reversed_and_lpt_bit_exact_with_timer():
    Hkv, G = 2, 4
    B = len(LENS)
    n = B * Hkv
    kc, vc, bt = make_paged(B, Hkv, LENS, seed=12)
    q = torch.randn(B, Hkv * G, 128, device=DEV).to(torch.bfloat16)
    stock, items = run_decode(q, kc, vc, bt, LENS)
    p = _plane(n)
    p.install_order(torch.arange(n - 1, -1, -1, dtype=torch.int32), n)
    p.set_timer_enabled(True)
    p.push()
    p.clear_timer()
    rev, _ = run_decode(q, kc, vc, bt, LENS, woven=True, slots=p.slots())
    assert torch.equal(stock, rev)
    cyc = p.read_timer()[:n]
    assert (cyc > 0).all(), "every task's timer row must be filled"
    # timer switched off -> rows stay zero; order_size mismatch -> identity (still exact)
    p.set_timer_enabled(False)
    p.set_order_size(n + 1)
    p.push()
    p.clear_timer()
    again, _ = run_decode(q, kc, vc, bt, LENS, woven=True, slots=p.slots())
    assert torch.equal(stock, again)
    assert int(p.read_timer()[:n].abs().sum()) == 0


def test_decode_shed_is_exact_truncated_softmax():
    Hkv, G = 2, 4
    B = len(LENS)
    n = B * Hkv
    kc, vc, bt = make_paged(B, Hkv, LENS, seed=13)
    q = torch.randn(B, Hkv * G, 128, device=DEV).to(torch.bfloat16)
    taus = [max(1, L // 2) for L in LENS]
    p = _plane(n)
    p.set_rows(tau=np.repeat(np.asarray(taus), Hkv), n=n)
    p.push()
    out, _ = run_decode(q, kc, vc, bt, LENS, woven=True, slots=p.slots())
    r = ref.decode_attention_paged(q, kc, vc, bt, LENS, 1 / math.sqrt(128), taus=taus)
    assert rel_err(out, r) < 2e-2


@pytest.mark.parametrize("acquire", [1, 2])
def test_decode_work_queue_bit_exact(acquire):
    Hkv, G = 8, 4
    lens = list(np.random.default_rng(5).integers(16, 4000, size=64))
    B = len(lens)
    n = B * Hkv
    kc, vc, bt = make_paged(B, Hkv, lens, seed=14)
    q = torch.randn(B, Hkv * G, 128, device=DEV).to(torch.bfloat16)
    stock, _ = run_decode(q, kc, vc, bt, lens)
    p = _plane(n)
    cost = torch.tensor([float(lens[t // Hkv]) for t in range(n)])
    p.install_order(p.region_order(cost, 148), n)
    p.set_num_tasks(n)
    p.set_timer_enabled(True)
    p.push()
    p.clear_timer()
    grid = 148 if acquire == 1 else 0
    for _ in range(3):  # repeated launches: the ticket queue resets itself
        out, _ = run_decode(q, kc, vc, bt, lens, woven=True, slots=p.slots(), acquire=acquire, grid=grid)
        assert torch.equal(stock, out)
    assert (p.read_timer()[:n] > 0).all()
    assert int(p.queue_t.abs().sum()) == 0


# ------------------------------------------------------------------ prefill attention
@pytest.mark.parametrize("qlens,prefix,Hkv,G", [
    ([1, 64, 65, 200], [0, 0, 0, 0], 2, 4),
    ([37, 128], [100, 16], 2, 4),
    ([129, 300, 7], [0, 257, 1000], 1, 8),      # unaligned prefixes, ragged last tiles
    ([1536], [0], 8, 4),                         # the named prompt: 12 tiles x 12 KV blocks
    ([256, 1], [2048, 4095], 2, 1),              # chunk after a long cached prefix; one-row decode-like tile
])
def test_prefill_attention(qlens, prefix, Hkv, G):
    """tcgen05 prefill attention against fp32 causal softmax attention, tiles
    of PREFILL_TILE_ROWS rows launched longest first, with empty tiles mixed in."""
    Hq, D = Hkv * G, 128
    R = ops.PREFILL_TILE_ROWS
    total = [q + p for q, p in zip(qlens, prefix)]
    kc, vc, bt = make_paged(len(qlens), Hkv, total, seed=21)
    Tq = sum(qlens)
    q = torch.randn(Tq, Hq, D, device=DEV).to(torch.bfloat16)
    tiles, row = [], 0
    for b, (ql, pf) in enumerate(zip(qlens, prefix)):
        for t0 in range(0, ql, R):
            tiles.append((b, row + t0, min(R, ql - t0), pf + t0))
        row += ql
    tiles.sort(key=lambda t: -(t[2] * (t[3] + t[2])))
    tiles.insert(1, (0, 0, 0, 0))  # an empty tile (graph padding) does nothing
    tt = torch.tensor(tiles, dtype=torch.int32, device=DEV)
    kvl = torch.tensor(total, dtype=torch.int32, device=DEV)
    out = torch.zeros_like(q)
    ops.attention_prefill(q, out, kc, vc, bt, kvl, tt, len(tiles), 1 / math.sqrt(D))
    torch.cuda.synchronize()
    row = 0
    for b, (ql, pf) in enumerate(zip(qlens, prefix)):
        k = ref.gather_kv(kc, bt[b], total[b])
        v = ref.gather_kv(vc, bt[b], total[b])
        r = ref.attention(q[row:row + ql], k, v, 1 / math.sqrt(D), causal_offset=pf)
        assert rel_err(out[row:row + ql], r) < 1e-2
        row += ql


def test_prefill_attention_rows_do_not_depend_on_the_tiling():
    """A prompt prefilled whole and the same prompt prefilled in two chunks
    (different 128-row tiles) give every row the same bits: a row's online
    softmax depends only on its own scores, so serving runs that chunk a
    prompt differently produce identical KV caches and tokens."""
    Hkv, G, D = 2, 4, 128
    L, cut = 300, 100
    kc, vc, bt = make_paged(1, Hkv, [L], seed=8)
    q = torch.randn(L, Hkv * G, D, device=DEV).to(torch.bfloat16)

    def run(chunks):
        out = torch.zeros_like(q)
        for q0, q1 in chunks:  # each chunk sees the cache up to its own end
            tiles = [(0, t0, min(128, q1 - t0), t0) for t0 in range(q0, q1, 128)]
            tt = torch.tensor(tiles, dtype=torch.int32, device=DEV)
            ops.attention_prefill(q, out, kc, vc, bt, torch.tensor([q1], dtype=torch.int32, device=DEV), tt,
                                  len(tiles), 1 / math.sqrt(D))
        torch.cuda.synchronize()
        return out
    whole = run([(0, L)])
    assert torch.equal(run([(0, cut), (cut, L)]), whole)
    assert torch.equal(run([(0, 7), (7, 200), (200, L)]), whole)


def test_prefill_attention_lazy_rescale():
    """Scores that grow by far more than 2^8 along the keys force the O
    rescale in TMEM on later blocks; the result is still exact softmax."""
    Hkv, G, D = 1, 2, 128
    L = 640
    kc, vc, bt = make_paged(1, Hkv, [L], seed=5)
    # key norms grow with position: each later block's max exceeds the last by >> 8 (log2)
    scale = torch.linspace(0.2, 6.0, L, device=DEV)
    k = ref.gather_kv(kc, bt[0], L).float()
    pages = bt[0, :(L + 15) // 16].long()
    kf = (k * scale[:, None, None]).to(torch.bfloat16)
    kc.view(-1, Hkv, 16, D)[pages] = kf.view(-1, 16, Hkv, D).transpose(1, 2).contiguous()
    q = (torch.randn(L, Hkv * G, D, device=DEV) * 2).to(torch.bfloat16)
    tiles = [(0, t0, min(128, L - t0), t0) for t0 in range(0, L, 128)][::-1]
    tt = torch.tensor(tiles, dtype=torch.int32, device=DEV)
    out = torch.zeros_like(q)
    ops.attention_prefill(q, out, kc, vc, bt, torch.tensor([L], dtype=torch.int32, device=DEV), tt,
                          len(tiles), 1 / math.sqrt(D))
    torch.cuda.synchronize()
    r = ref.attention(q, ref.gather_kv(kc, bt[0], L), ref.gather_kv(vc, bt[0], L), 1 / math.sqrt(D),
                      causal_offset=0)
    assert torch.isfinite(out.float()).all()
    assert rel_err(out, r) < 1e-2


@pytest.mark.parametrize("T,N,K,grid", [
    (1, 4096, 4096, 0), (6, 4096, 4096, 0), (16, 4096, 14336, 0), (6, 4096, 4096, 148),
    (100, 4096, 4096, 0), (300, 4096, 14336, 0), (1541, 4096, 4096, 0), (6, 8192, 1024, 0), (5, 12288, 512, 0),
])
def test_linear_add_rmsnorm_fused_matches_separate_kernels(T, N, K, grid, monkeypatch):
    """The projection with the residual add + RMSNorm in its epilogue gives
    the same bits as the GEMM followed by add_rmsnorm (cluster split-K and
    stream-K schedules, hidden sizes using 256, 512 and 1024 virtual norm
    threads), twice in a row (the row counters reset themselves). The plain
    GEMM is held on the single-CTA schedules the fused one uses (the CTA-pair
    schedule sums K in another order)."""
    monkeypatch.setenv("SCHED_GEMM_PAIR", "0")
    g = torch.Generator(device="cuda").manual_seed(T + N + K)
    x = torch.randn(T, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    res0 = torch.randn(T, N, device="cuda", generator=g).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(N, device="cuda", generator=g)).to(torch.bfloat16)
    y1 = ops.linear(x, w, grid=grid)
    r1 = res0.clone()
    n1 = ops.add_rmsnorm(y1, r1, nw, 1e-5)
    for _ in range(2):
        y2 = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
        r2 = res0.clone()
        n2 = torch.empty_like(r2)
        ops.linear_add_rmsnorm(x, w, y2, r2, nw, 1e-5, n2, grid=grid)
        torch.cuda.synchronize()
        ops.check_status()
        assert torch.equal(y2, y1) and torch.equal(r2, r1) and torch.equal(n2, n1)
    assert int(ops.kernels.row_counters(x.device, T)[:T].abs().sum()) == 0
