"""The sequence-parallel kernels with W emulated ranks on one GPU.

Rank r's buffers are ordinary device tensors of this process and every
"peer pointer" is another rank's tensor, so the multi-rank index arithmetic
(row ownership, per-source row-flag offsets, all-gather into every rank's
buffer, per-rank ready flags) runs for real. The launches go rank by rank and
phase by phase -- every reduce-scatter GEMM, then every owner's norm, then
every ready-gated GEMM -- so each kernel finds the flags it waits for
already raised by kernels that completed before it: no launch waits on a
later one.

Checked bit for bit against the single-GPU reference of the same arithmetic:
the partial products (``ops.linear``) summed in rank order in fp32 and
rounded once (the fused all-reduce's value), then ``ops.add_rmsnorm``; the
ready-gated GEMM against the ungated one. Also: flags are left clean for the
next call (second call on the same buffers), and a ready flag that nothing
raises ends in a peer-timeout status instead of a hang.
"""
import math
import time

import pytest
import torch

from sched_pass_b200 import ops
from sched_pass_b200._ext import ext
from sched_pass_b200.ops.kernels import STATUS_NAMES
from sched_pass_b200.parallel.sp import owned_rows

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _single_cta_gemm_schedules(monkeypatch):
    """The reference products use ops.linear, checked bit for bit against the
    reduce-scatter and ready-gated GEMMs, which run the single-CTA schedules;
    hold ops.linear on them too (the CTA-pair schedule sums K in another order)."""
    monkeypatch.setenv("SCHED_GEMM_PAIR", "0")

EPS = 1e-5


def bits(t):
    return t.contiguous().view(torch.int16)


class Ranks:
    """Per-rank buffers: receive slab [W, M, H], row flags [W * H/128 * M],
    two gather sets [M, H] with ready flags [M]."""

    def __init__(self, W, M, H, dev="cuda"):
        self.W, self.M, self.H = W, M, H
        z = lambda *s, dt=torch.bfloat16: torch.zeros(*s, dtype=dt, device=dev)  # noqa: E731
        self.slab = [z(W, M, H) for _ in range(W)]
        self.rflags = [z(W * (H // 128) * M, dt=torch.int32) for _ in range(W)]
        self.gather = [[z(M, H) for _ in range(W)] for _ in range(2)]
        self.ready = [[z(M, dt=torch.int32) for _ in range(W)] for _ in range(2)]

    def ptrs(self, lst):
        return [t.data_ptr() for t in lst]


def sublayer(R, xs, ws, res, lnw, g, T, status):
    """GEMM -> reduce-scatter for every rank, then every owner's norm (gather
    set g; clears set g^1), then returns the per-rank gathered views."""
    W = R.W
    for r in range(W):
        ws_ = ops.kernels._ws_for(xs[r], ws[r].shape[0], xs[r].shape[1], 0, None)
        ext().gemm_reduce_scatter(xs[r], ws[r], r, W, R.ptrs(R.slab), R.ptrs(R.rflags), 0, ws_.ws,
                                  ws_.counters, status)
    deltas = []
    for r in range(W):
        d = torch.zeros(T, R.H, dtype=torch.bfloat16, device="cuda")
        ext().sp_reduce_norm(R.slab[r].data_ptr(), R.rflags[r].data_ptr(), res[r], lnw, d,
                             R.ptrs(R.gather[g]), R.ptrs(R.ready[g]), R.ready[g ^ 1][r].data_ptr(), R.M, T, r, W,
                             EPS, status)
        deltas.append(d)
    return [R.gather[g][r][:T] for r in range(W)], deltas


@pytest.mark.parametrize("W", [1, 2, 3, 4])
def test_sp_sublayer_matches_the_allreduce_arithmetic(W):
    torch.manual_seed(W)
    H, K, M = 1024, 256, 320
    R = Ranks(W, M, H)
    st = ops.status_buffer()
    lnw = (1 + 0.1 * torch.randn(H, device="cuda")).to(torch.bfloat16)
    w2 = (torch.randn(384, H, device="cuda") / math.sqrt(H)).to(torch.bfloat16)
    # second use of each set; shrinking and growing T; fewer rows than ranks (T = 1, 2)
    for call, T in enumerate([37, 300, 5, 1, 16, 2, 300]):
        g = call % 2
        xs = [torch.randn(T, K, device="cuda").to(torch.bfloat16) for _ in range(W)]
        wts = [(torch.randn(H, K, device="cuda") / math.sqrt(K * W)).to(torch.bfloat16) for _ in range(W)]
        res0 = torch.randn(T, H, device="cuda").to(torch.bfloat16)
        res = [res0.clone() for _ in range(W)]
        gathered, deltas = sublayer(R, xs, wts, res, lnw, g, T, st)
        # every rank's ready-gated GEMM on its gathered copy
        z = [ops.linear(gathered[r], w2, x_ready=R.ready[g][r].data_ptr()) for r in range(W)]
        torch.cuda.synchronize()
        ops.check_status()
        # reference: rank-order fp32 sum of the bf16 partials, rounded once; then add + RMSNorm
        acc = torch.zeros(T, H, dtype=torch.float32, device="cuda")
        for r in range(W):
            acc = acc + ops.linear(xs[r], wts[r]).float()
        delta = acc.to(torch.bfloat16)
        res_ref = res0.clone()
        normed = ops.add_rmsnorm(delta, res_ref, lnw, EPS)
        z_ref = ops.linear(normed, w2)
        for r in range(W):
            lo, hi = owned_rows(r, W, T)
            assert torch.equal(bits(deltas[r][lo:hi]), bits(delta[lo:hi])), (W, T, r, "delta")
            assert torch.equal(bits(res[r][lo:hi]), bits(res_ref[lo:hi])), (W, T, r, "residual")
            assert torch.equal(bits(gathered[r]), bits(normed)), (W, T, r, "gathered")
            assert torch.equal(bits(z[r]), bits(z_ref)), (W, T, r, "gated gemm")
        # consumed row flags are reset by their owners
        assert all(int(f.abs().sum()) == 0 for f in R.rflags), (W, T)


def test_gated_gemm_times_out_on_a_row_nothing_raises():
    """A ready flag that no owner raises: the GEMM's producer gives up after
    its wait budget, reports peer-timeout, and the kernel completes."""
    ops.check_status()
    x = torch.randn(40, 256, device="cuda").to(torch.bfloat16)
    w = torch.randn(256, 256, device="cuda").to(torch.bfloat16)
    ready = torch.ones(64, dtype=torch.int32, device="cuda")
    ready[33] = 0  # row 33 never arrives
    st = ops.status_buffer()
    t0 = time.perf_counter()
    ops.linear(x, w, x_ready=ready.data_ptr())
    torch.cuda.synchronize()
    assert STATUS_NAMES.get(int(st[0].item())) == "peer-timeout"
    assert time.perf_counter() - t0 < 30
    st.zero_()
    ops.check_status()
    # with every flag raised the same call completes cleanly and equals the ungated GEMM
    ready[33] = 1
    y1 = ops.linear(x, w, x_ready=ready.data_ptr())
    y2 = ops.linear(x, w)
    torch.cuda.synchronize()
    ops.check_status()
    assert torch.equal(bits(y1), bits(y2))


def test_sp_norm_times_out_on_a_missing_partial():
    """The owner's norm waits for every source's row flags; a source that
    never pushed ends in peer-timeout, not a hang."""
    ops.check_status()
    W, M, H, T = 2, 16, 256, 4
    R = Ranks(W, M, H)
    st = ops.status_buffer()
    res = torch.zeros(T, H, dtype=torch.bfloat16, device="cuda")
    lnw = torch.ones(H, dtype=torch.bfloat16, device="cuda")
    t0 = time.perf_counter()
    # rank 1 owns rows 2..3; nobody pushed: its flags stay 0
    ext().sp_reduce_norm(R.slab[1].data_ptr(), R.rflags[1].data_ptr(), res, lnw, None, R.ptrs(R.gather[0]),
                         R.ptrs(R.ready[0]), R.ready[1][1].data_ptr(), M, T, 1, W, EPS, st)
    torch.cuda.synchronize()
    assert STATUS_NAMES.get(int(st[0].item())) == "peer-timeout"
    assert time.perf_counter() - t0 < 30
    st.zero_()
    ops.check_status()
