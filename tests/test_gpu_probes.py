"""The lever probes: every acquisition mode runs each task exactly once, and
the cache-policy stream reads at a sane fraction of HBM bandwidth."""
import numpy as np
import pytest
import torch

from sched_pass_b200 import ops
from sched_pass_b200._ext import ext

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("memory", [False, True])
def test_task_probe_exactly_once(mode, memory):
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    R = ext().probe_tasks_occupancy() * sms
    n = 3 * R + 17
    rng = np.random.default_rng(mode)
    cost = rng.integers(1000, 20000, size=n) if not memory else np.full(n, 4096)
    c = torch.from_numpy(cost.astype(np.int32)).cuda()
    hits = torch.zeros(n, dtype=torch.int32, device="cuda")
    per = torch.zeros(max(n, R), dtype=torch.int32, device="cuda")
    ticket = torch.zeros(1, dtype=torch.int32, device="cuda")
    sink = torch.zeros(4, dtype=torch.int32, device="cuda")
    data = torch.zeros(1 << 22, dtype=torch.int32, device="cuda")
    ext().probe_tasks(c, mode, R, int(memory), data, hits, per, ticket, sink, ops.status_buffer())
    torch.cuda.synchronize()
    ops.check_status()
    assert (hits == 1).all()
    assert int(per.sum()) == n


def test_stream_probe_policies():
    src = torch.zeros(1 << 28, dtype=torch.int32, device="cuda")  # 1 GiB
    sink = torch.zeros(1 << 12, dtype=torch.int32, device="cuda")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for pol in range(5):
        ext().probe_stream(src, pol, sink, sms * 4)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ext().probe_stream(src, pol, sink, sms * 4)
        b.record()
        b.synchronize()
        gbs = src.numel() * 4 / a.elapsed_time(b) / 1e6
        assert gbs > 1000, (pol, gbs)
