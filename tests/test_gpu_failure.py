"""Device-side bounded waits that run out on purpose: a flag that nothing
sets makes the kernel report a peer timeout in the status word and return;
the context stays usable. (No fault, trap or hang is involved.)"""
import time

import pytest
import torch

from sched_pass_b200 import ops
from sched_pass_b200._ext import ext
from sched_pass_b200.ops.kernels import STATUS_NAMES

pytestmark = pytest.mark.gpu


def test_combine_wait_for_missing_rows_times_out_with_status():
    ops.check_status()
    T, K, H = 2, 2, 512
    c = torch.zeros(T * K, H, dtype=torch.bfloat16, device="cuda")
    h = torch.randn(T, H, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(H, dtype=torch.bfloat16, device="cuda")
    y = torch.empty_like(h)
    words = torch.zeros(8, dtype=torch.int32, device="cuda")  # cnt stays 0: the rows never arrive
    base = words.data_ptr()
    st = ops.status_buffer()
    t0 = time.perf_counter()
    ext().moe_combine_norm(c.data_ptr(), K, h, w, y, T, 1e-5, base, base + 4, base + 8, st)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    code = int(st[0].item())
    assert STATUS_NAMES.get(code) == "peer-timeout", code
    assert dt < 30
    st.zero_()
    # the context still works
    z = torch.randn(64, 64, device="cuda")
    assert torch.allclose(z @ torch.eye(64, device="cuda"), z)
    ops.check_status()


def test_expert_gemm_wait_for_absent_sources_times_out():
    from sched_pass_b200.models.config import MIXTRAL_TINY
    from sched_pass_b200.parallel.ep import ExpertParallel, build_moe_weights
    cfg = MIXTRAL_TINY
    ep = ExpertParallel(cfg, "cuda", max_tokens=8)
    g = torch.Generator(device="cuda").manual_seed(0)
    w = build_moe_weights(cfg, 0, 1, g, "cuda")
    st = ops.status_buffer()
    # no dispatch ran: the owner's done count never reaches the world size
    ext().moe_expert_gemm(0, w.w13, ep.mine("slab"), ep.E_local, 2 * ep.I, ep.H, ep.rows, w.s13,
                          ep.mine("slab_scale"), ep.act.data_ptr(), ep.mine("counter"), ep.mine("done"),
                          ep.rows_valid, ep.tiles_done, 1, ep.capacity, ep.mine("slab_meta"), [], [], ep.K,
                          ep.ws.data_ptr(), ep.tile_counters.data_ptr(), ep.grid, 0, st)
    torch.cuda.synchronize()
    assert STATUS_NAMES.get(int(st[0].item())) == "peer-timeout"
    st.zero_()
    ep.close()
    ops.check_status()
