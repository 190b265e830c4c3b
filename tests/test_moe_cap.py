"""The capacity lever as a routing-tensor function (GPU-free)."""
import torch

from sched_pass_b200.parallel.ep import dequantize_blockwise_fp8, moe_expert_cap, quantize_blockwise_fp8


def test_cap_drops_exactly_the_overflow():
    NT, K, E = 1024, 2, 16
    g = torch.Generator().manual_seed(0)
    ti = torch.randint(0, E, (NT, K), generator=g)
    ti[: int(0.4 * NT), 0] = 0  # a hot expert
    tw = torch.rand(NT, K, generator=g)
    counts = torch.bincount(ti.reshape(-1), minlength=E)
    w, dropped = moe_expert_cap(ti, tw, E, capacity_factor=1.25)
    C = int(1.25 * NT * K / E)
    assert dropped == int((counts - C).clamp_min(0).sum())
    assert int((w.reshape(-1)[ti.reshape(-1) == 0] > 0).sum()) == C
    assert int((w > 0).sum()) == NT * K - dropped
    # arrival order: the first C assignments of the hot expert are kept
    flat = ti.reshape(-1)
    kept = (w.reshape(-1) > 0) & (flat == 0)
    first = torch.nonzero(flat == 0).flatten()[:C]
    assert kept[first].all()


def test_cap_balanced_and_small_batches_are_noops():
    NT, K, E = 1024, 2, 16
    tw = torch.rand(NT, K)
    tib = torch.arange(NT * K).reshape(NT, K) % E
    w, d = moe_expert_cap(tib, tw, E, 1.25)
    assert d == 0 and torch.equal(w, tw)
    tid = torch.randint(0, 128, (16, 8))
    w2, d2 = moe_expert_cap(tid, torch.rand(16, 8), 128, capacity_factor=1.0)
    assert d2 == 0


def test_blockwise_fp8_roundtrip():
    w = torch.randn(256, 384)
    q, s = quantize_blockwise_fp8(w)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (2, 3)
    r = dequantize_blockwise_fp8(q, s)
    assert ((r - w).norm() / w.norm()).item() < 0.05
