"""IR-woven kernels on the B200: hand-written NVPTX fixtures, woven by
sched-weave, compiled by LLVM's NVPTX backend for sm_100a and loaded through
the driver, run in each lever mode against the unwoven kernel.

Modes (as the reference's host fixtures): A inert (slots null) bit-exact;
B identity order + timer rows filled; C reversed pi bit-exact; D aggressive
policy (every task urgent / polite) bit-exact; G shed tau = 0 bit-exact and
tau > 0 = truncated softmax; work queue with ticket (W < tasks) and with
cluster launch control (grid = tasks), bit-exact; num_tasks = 0 disarms the
claim loop."""
import math
import os
import struct

import numpy as np
import pytest
import torch

from sched_pass_b200.runtime import abi

pytestmark = pytest.mark.gpu
HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ir")
B, G, D, PS = 8, 4, 64, 16


def _compile(name, env=None):
    from sched_pass_b200.compiler.nvptx import CudaModule, compile_ptx
    from sched_pass_b200.compiler.weave import weave
    src = open(os.path.join(HERE, name)).read()
    if env is not None:
        if env.get("SCHED_WORKQUEUE") and not env.get("SCHED_CLC"):
            src = src.replace("@__sched_timer = ", "@__sched_queue = addrspace(1) externally_initialized "
                                                   "global ptr null, align 8\n@__sched_timer = ")
        src, _ = weave(src, env)
    return CudaModule(compile_ptx(src))


class Tables:
    def __init__(self, n=1024):
        self.n = n
        self.order = torch.arange(n, dtype=torch.int32, device="cuda")
        self.host = bytearray(abi.ctrl_bytes(n))
        self.ctrl = torch.zeros(abi.ctrl_bytes(n), dtype=torch.uint8, device="cuda")
        self.timer = torch.zeros(n, dtype=torch.int64, device="cuda")
        self.queue = torch.zeros(4, dtype=torch.int32, device="cuda")

    def row(self, i, q=0.0, tau=0, hint=0):
        struct.pack_into("<fHB", self.host, abi.CTRL_ROWS_OFF + abi.ROW_SIZE * i, q, tau, hint)

    def u32(self, off, v):
        struct.pack_into("<I", self.host, off, v)

    def push(self):
        self.ctrl.copy_(torch.frombuffer(bytearray(self.host), dtype=torch.uint8))

    def arm(self, mod, queue=False):
        mod.set_global_ptr("__sched_task_order", self.order.data_ptr())
        mod.set_global_ptr("__sched_ctrl", self.ctrl.data_ptr())
        mod.set_global_ptr("__sched_timer", self.timer.data_ptr())
        if queue:
            mod.set_global_ptr("__sched_queue", self.queue.data_ptr())

    @staticmethod
    def disarm(mod, queue=False):
        for g in ("__sched_task_order", "__sched_ctrl", "__sched_timer") + (("__sched_queue",) if queue else ()):
            mod.set_global_ptr(g, 0)


def softmax_inputs(seed=0, nreq=B):
    rng = np.random.default_rng(seed)
    lens = rng.integers(16, 513, size=nreq).astype(np.int32)
    npg = (lens + PS - 1) // PS
    total = int(npg.sum())
    perm = rng.permutation(total).astype(np.int32)
    maxp = int(npg.max())
    bt = np.zeros((nreq, maxp), np.int32)
    k = 0
    for b in range(nreq):
        bt[b, :npg[b]] = perm[k:k + npg[b]]
        k += npg[b]
    t = lambda a: torch.from_numpy(a).cuda()
    kc = torch.randn(total, PS, D, device="cuda")
    vc = torch.randn(total, PS, D, device="cuda")
    q = torch.randn(nreq, G, D, device="cuda")
    return dict(lens=t(lens), bt=t(bt), kc=kc, vc=vc, q=q, maxp=maxp, lens_np=lens, bt_np=bt)


def run_softmax(mod, x, grid=None):
    nreq = x["q"].shape[0]
    out = torch.zeros_like(x["q"])
    acc = torch.zeros_like(x["q"])
    mod.launch("softmax_decode", (grid or nreq,), (G,),
               [x["q"], x["kc"], x["vc"], x["bt"], x["lens"], out, acc, x["maxp"], G,
                math.log2(math.e) / math.sqrt(D)])
    torch.cuda.synchronize()
    return out


def softmax_ref(x, taus=None):
    out = torch.zeros_like(x["q"], dtype=torch.float64)
    for b in range(x["q"].shape[0]):
        n = int(x["lens_np"][b])
        if taus is not None and taus[b] > 0:
            n = min(n, int(taus[b]))
        pages = torch.from_numpy(x["bt_np"][b, :(int(x["lens_np"][b]) + PS - 1) // PS]).long().cuda()
        K = x["kc"][pages].reshape(-1, D)[:n].double()
        V = x["vc"][pages].reshape(-1, D)[:n].double()
        s = (K @ x["q"][b].double().t()).t() / math.sqrt(D)
        out[b] = torch.softmax(s, -1) @ V
    return out.float()


def test_softmax_fixture_modes():
    stock = _compile("softmax_decode.ll")
    woven = _compile("softmax_decode.ll", {})
    x = softmax_inputs(0)
    base = run_softmax(stock, x)
    assert (base - softmax_ref(x)).abs().max().item() < 1e-3
    # A: inert (null slots)
    Tables.disarm(woven)
    assert torch.equal(run_softmax(woven, x), base)
    t = Tables()
    t.push()
    t.arm(woven)
    # B: identity + timer
    t.timer.zero_()
    assert torch.equal(run_softmax(woven, x), base)
    assert (t.timer[:B] > 0).all()
    # C: reversed pi (order_size stamped)
    t.order[:B] = torch.arange(B - 1, -1, -1, dtype=torch.int32, device="cuda")
    t.u32(abi.CTRL_ORDER_SIZE_OFF, B)
    t.push()
    assert torch.equal(run_softmax(woven, x), base)
    # D: aggressive policy (all urgent, then all polite) -- hints only
    for hint in (abi.HINT_URGENT, abi.HINT_POLITE):
        for b in range(B):
            t.row(b, q=1.0, hint=hint)
        t.push()
        assert torch.equal(run_softmax(woven, x), base)
    # G: shed -- tau = 0 bit-exact, tau > 0 exact truncated softmax
    taus = [max(1, int(n) // 2) for n in x["lens_np"]]
    for b in range(B):
        t.row(b, tau=0)
    t.push()
    assert torch.equal(run_softmax(woven, x), base)
    for b in range(B):
        t.row(b, tau=taus[b])
    t.push()
    # reversed order: the tau of task i applies to request i
    shed = run_softmax(woven, x)
    assert (shed - softmax_ref(x, taus)).abs().max().item() < 1e-3
    assert not torch.equal(shed, base)


@pytest.mark.parametrize("clc", [False, True])
def test_softmax_fixture_work_queue(clc):
    nreq = 64
    stock = _compile("softmax_decode.ll")
    env = {"SCHED_WORKQUEUE": "1"}
    if clc:
        env["SCHED_CLC"] = "1"
    wq = _compile("softmax_decode.ll", env)
    x = softmax_inputs(3, nreq)
    base = run_softmax(stock, x)
    t = Tables()
    t.push()
    t.arm(wq, queue=not clc)
    # num_tasks = 0: stock path (grid = tasks), bit-exact
    assert torch.equal(run_softmax(wq, x), base)
    # claim loop on, LPT order by length
    order = np.argsort(-x["lens_np"], kind="stable").astype(np.int32)
    t.order[:nreq] = torch.from_numpy(order).cuda()
    t.u32(abi.CTRL_ORDER_SIZE_OFF, nreq)
    t.u32(abi.CTRL_NUM_TASKS_OFF, nreq)
    t.push()
    workers = 16
    for _ in range(3):
        t.timer.zero_()
        if not clc:
            t.queue[0] = workers  # reference semantics: prime the ticket to the worker count
        out = run_softmax(wq, x, grid=workers if not clc else nreq)
        assert torch.equal(out, base)
        assert (t.timer[:nreq] > 0).all()


def test_paged_linear_fixture():
    stock = _compile("paged_linear.ll")
    woven = _compile("paged_linear.ll", {})
    nreq, nb = 32, 24
    kv = torch.randn(nreq * nb * 64, device="cuda")
    bt = torch.randperm(nreq * nb, device="cuda").to(torch.int32)
    w = torch.randn(nb, device="cuda")

    def run(mod):
        out = torch.zeros(nreq * 64, device="cuda")
        mod.launch("paged_linear", (nreq,), (64,), [kv, bt, w, out, nb])
        torch.cuda.synchronize()
        return out
    base = run(stock)
    ref = (kv.view(-1, 64)[bt.view(nreq, nb).long()] * w[None, :, None]).sum(1).flatten()
    assert (base - ref).abs().max().item() < 1e-3
    Tables.disarm(woven)
    assert torch.equal(run(woven), base)
    t = Tables()
    t.order[:nreq] = torch.arange(nreq - 1, -1, -1, dtype=torch.int32, device="cuda")
    t.u32(abi.CTRL_ORDER_SIZE_OFF, nreq)
    t.push()
    t.arm(woven)
    assert torch.equal(run(woven), base)
    for b in range(nreq):
        t.row(b, tau=nb // 2)
    t.push()
    shed = run(woven)
    ref_half = (kv.view(-1, 64)[bt.view(nreq, nb)[:, :nb // 2].long()] * w[None, :nb // 2, None]).sum(1).flatten()
    assert (shed - ref_half).abs().max().item() < 1e-3


def test_paged_linear_pdl_after_producer():
    """PDL lever: the woven consumer, launched with programmatic stream
    serialization right behind a kernel that writes its KV (and releases its
    dependents at entry), reads only finished data -- the same bits as a
    plain launch -- and its woven timer still fills."""
    from sched_pass_b200._ext import ext
    woven = _compile("paged_linear.ll", {"SCHED_PDL": "1"})
    nreq, nb = 32, 24
    kv = torch.empty(nreq * nb * 64, device="cuda")
    bt = torch.randperm(nreq * nb, device="cuda").to(torch.int32)
    w = torch.randn(nb, device="cuda")
    t = Tables()
    t.u32(abi.CTRL_ORDER_SIZE_OFF, nreq)
    t.push()
    t.arm(woven)

    def run(pdl):
        out = torch.zeros(nreq * 64, device="cuda")
        kv.zero_()
        t.timer.zero_()
        ext().probe_pdl_produce(kv, 2048)  # a long producer: the consumer would see zeros if it ran early
        woven.launch("paged_linear", (nreq,), (64,), [kv, bt, w, out, nb], pdl=pdl)
        torch.cuda.synchronize()
        return out
    plain = run(False)
    got = run(True)
    assert torch.equal(got, plain)
    ref = (kv.view(-1, 64)[bt.view(nreq, nb).long()] * w[None, :, None]).sum(1).flatten()
    assert (got - ref).abs().max().item() < 1e-3 and kv.abs().sum().item() > 0
    assert (t.timer[:nreq] > 0).all()


def test_hetero_batch_closed_loop():
    """The reference's heterogeneous batch (8 long + 56 short requests, 16
    ticket workers): every arm is bit-exact with the stock launch, the woven
    timer ranks the long requests costliest, and LPT from those cycles does
    not lose to the identity order."""
    from sched_pass_b200.benchmarks import hetero_batch
    rec = hetero_batch.run(iters=5, emit=lambda s: None)
    assert all(rec["bit_exact"].values()), rec
    assert rec["timer_ranks_longs_first"], rec
    assert rec["lpt_us"] <= 1.1 * rec["identity_us"], rec
