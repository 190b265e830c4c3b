"""Tiered KV bookkeeping on the CPU: spill order (never-read pages first,
then least urgent), the appended page stays on the device, staging slots
and the published copy pairs, host pages returned on release. The page
copies run as torch copies here (the CUDA kernel and the per-layer
streaming are covered by the GPU tests)."""
import numpy as np
import pytest
import torch

from sched_pass_b200.engine.request import Request, State
from sched_pass_b200.engine.scheduler import Scheduler
from sched_pass_b200.engine.tiered_kv import HOST_BASE, TieredKV, is_host
from sched_pass_b200.models.config import LLAMA_TINY
from sched_pass_b200.models.llama import KVCache


def cpu_copy(src_k, src_v, dst_k, dst_v, pairs):
    for s, d in pairs:
        dst_k[:, d] = src_k[:, s]
        dst_v[:, d] = src_v[:, s]


def make(n_device=40, n_staging=16, n_host=64):
    kv = KVCache(LLAMA_TINY, n_device, "cpu")
    kv.k.copy_(torch.arange(kv.k.numel(), dtype=torch.float32).reshape(kv.k.shape).to(torch.bfloat16))
    kv.v.copy_(-kv.k)
    tier = TieredKV(kv, n_device, n_staging, n_host, "cpu")
    tier._copy_all_layers = cpu_copy
    sched = Scheduler(n_device, 16, 8, 256, 4096, tier=tier)
    return kv, tier, sched


def admit(sched, rid, n_tokens, urgency, tau=0):
    r = Request(rid=rid, prompt=np.zeros(n_tokens, dtype=np.int32), max_new_tokens=64, urgency=urgency, tau=tau)
    sched.admit_cached(r, 1, 0.0)
    return r


def test_spill_prefers_never_read_pages_then_least_urgent():
    kv, tier, sched = make(n_device=40)
    a = admit(sched, 0, 16 * 12, urgency=0.9)            # 12 pages, urgent
    b = admit(sched, 1, 16 * 12, urgency=0.1, tau=16 * 4)  # least urgent, reads 4 pages only
    c = admit(sched, 2, 16 * 12, urgency=0.5)            # 36 pages used, 4 free
    before_b = kv.k[:, b.pages[5]].clone()
    d = admit(sched, 3, 16 * 10, urgency=0.7)            # needs 10 -> 6 spilled
    assert sched.alloc.free >= 0 and len(d.pages) == 10
    spilled_b = [i for i, p in enumerate(b.pages) if is_host(p)]
    assert spilled_b == [4, 5, 6, 7, 8, 9]               # beyond its horizon, oldest first
    assert not any(is_host(p) for p in a.pages + c.pages + d.pages)
    assert torch.equal(tier.host_k[:, b.pages[5] - HOST_BASE], before_b)  # data moved intact
    assert tier.spilled_pages == 6


def test_last_page_and_urgent_requests_are_protected():
    kv, tier, sched = make(n_device=30)
    a = admit(sched, 0, 16 * 14, urgency=0.9)
    b = admit(sched, 1, 16 * 14, urgency=0.2)
    admit(sched, 2, 16 * 8, urgency=0.5)
    assert not is_host(b.pages[-1]) and not is_host(a.pages[-1])
    assert any(is_host(p) for p in b.pages) and not any(is_host(p) for p in a.pages)


def test_stage_translates_read_pages_and_release_returns_host_pages():
    kv, tier, sched = make(n_device=40, n_staging=16)
    a = admit(sched, 0, 16 * 12, urgency=0.9)
    b = admit(sched, 1, 16 * 12, urgency=0.1)
    admit(sched, 2, 16 * 12, urgency=0.5)
    admit(sched, 3, 16 * 10, urgency=0.7)
    host_idx = [i for i, p in enumerate(b.pages) if is_host(p)]
    assert host_idx
    tier.stage([a, b])
    tr = tier.pages_for(b)
    # what the page-copy kernels read: the count and the (host page, slot) pairs on the device
    n = int(tier.count_dev[0])
    pairs = tier.pairs_dev[: 2 * n].numpy()
    assert n == len(host_idx) and tier.last_stage == n
    got = {int(pairs[1 + 2 * j]): int(pairs[2 * j]) for j in range(n)}  # slot -> host page
    for i in host_idx:
        slot = tr[i] - tier.split
        assert tier.split == 40 and 0 <= slot < 16
        assert got[slot] == b.pages[i] - HOST_BASE
    assert tier.pages_for(a) == a.pages
    free0 = tier.host_free
    b.state = State.DONE
    sched.release(b)
    assert tier.host_free == free0 + len(host_idx)


def test_staging_overflow_is_loud():
    kv, tier, sched = make(n_device=40, n_staging=2)
    admit(sched, 0, 16 * 12, urgency=0.9)
    b = admit(sched, 1, 16 * 12, urgency=0.1)
    admit(sched, 2, 16 * 12, urgency=0.5)
    admit(sched, 3, 16 * 10, urgency=0.7)
    with pytest.raises(RuntimeError, match="staging"):
        tier.stage([b])


def test_staged_pages_coalesce_into_contiguous_runs():
    from sched_pass_b200.engine.tiered_kv import coalesce_runs
    pairs = [(5, 0), (6, 1), (7, 2), (2, 3), (9, 4), (10, 5), (12, 6)]
    assert coalesce_runs(pairs) == [(5, 0, 3), (2, 3, 1), (9, 4, 2), (12, 6, 1)]
    assert coalesce_runs([]) == []


def test_consecutive_steps_publish_each_steps_pairs():
    """Staging alternates between two pinned upload buffers (a buffer is
    reused only after its upload of two steps ago), and every step publishes
    its own pairs: a step that reads fewer host pages after one that read
    more leaves the device count and pairs of the smaller step."""
    kv, tier, sched = make(n_device=40, n_staging=16)
    a = admit(sched, 0, 16 * 12, urgency=0.9)
    b = admit(sched, 1, 16 * 12, urgency=0.1)
    admit(sched, 2, 16 * 12, urgency=0.5)
    admit(sched, 3, 16 * 10, urgency=0.7)
    host_b = [p - HOST_BASE for p in b.pages if is_host(p)]
    assert len(host_b) >= 2
    published = []
    for step, reqs in enumerate([[a, b], [a], [a, b]]):
        tier.stage(reqs)
        n = int(tier.count_dev[0])
        pairs = tier.pairs_dev[: 2 * n].numpy().reshape(-1, 2)
        published.append(sorted(int(h) for h, _ in pairs))
        assert tier._pin_k == (step + 1) % 2
    assert published == [sorted(host_b), [], sorted(host_b)]
