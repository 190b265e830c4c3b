"""The IR weaver on hand-written NVPTX fixtures (GPU-free): structure of the
woven code (FileCheck-style ordered patterns), knob gating, verification by
LLVM's own parser/verifier, and the manifest mirror."""
import os
import re

import pytest

from sched_pass_b200.compiler.weave import manifest_csv, weave
from sched_pass_b200.runtime.manifest import MANIFEST

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ir")


def fixture(name):
    with open(os.path.join(HERE, name)) as f:
        return f.read()


def check_order(text, patterns):
    """Each regex must match, in order, after the previous match."""
    pos = 0
    for p in patterns:
        m = re.compile(p, re.M).search(text, pos)
        assert m, f"pattern not found after offset {pos}: {p}"
        pos = m.end()


def verify(text):
    import llvmlite.binding as llvm
    llvm.initialize_all_targets()
    llvm.initialize_all_asmprinters()
    m = llvm.parse_assembly(text)
    m.verify()


def test_weave_paged_linear_structure():
    out, notes = weave(fixture("paged_linear.ll"))
    verify(out)
    check_order(out, [
        r"define ptx_kernel void @paged_linear\(.*\"sched-instrumented\"",
        # timer: clock at entry, off-flag latched at entry, gated on ctrl armed
        r"%sched\.t0 = call i64 @llvm\.nvvm\.read\.ptx\.sreg\.clock64\(\)",
        r"%sched\.flags = load i32",
        r"%sched\.timer\.off = icmp ne i32",
        r"%sched\.timer\.gate = select i1 %sched\.ctrl\.armed",
        # pi: armed + bounds guard, table load, order_size validity, clamp, select
        r"%sched\.pid = call i32 @llvm\.nvvm\.read\.ptx\.sreg\.ctaid\.x\(\)",
        r"%sched\.order\.use = and i1 %sched\.task_order\.armed, %sched\.pid\.inb",
        r"%sched\.task\.mapped = load i32",
        r"%sched\.order\.size = load i32",
        r"%sched\.order\.valid = or i1",
        r"%sched\.order\.szok = and i1",
        r"%sched\.task\.ingrid = icmp ult i32 %sched\.task\.mapped, %sched\.ntiles",
        r"%sched\.task\.ok = and i1 %sched\.task\.ingrid, %sched\.order\.szok",
        r"%sched\.task = select i1 %sched\.task\.ok, i32 %sched\.task\.mapped, i32 %sched\.pid",
        # the original ctaid use now reads the remapped task
        r"%row = mul i32 %sched\.task, %nb",
        # shed on the canonical IV %i, value mask after the stream load
        r"%v = load float",
        r"%sched\.keep(\.\d+)? = icmp ult i32 %i, %sched\.budget",
        r"select i1 %sched\.keep(\.\d+)?, float %v, float 0\.000000e\+00",
        # timer at the return: cycles, gate, guarded monotonic atomic add
        r"%sched\.cycles = sub i64 %sched\.t1, %sched\.t0",
        r"%sched\.timer\.on = xor i1 %sched\.timer\.gate, true",
        r"br i1 %sched\.timer\.ok, label %sched\.timer\.do, label %sched\.timer\.ret",
        r"atomicrmw add ptr %sched\.timer\.row, i64 %sched\.cycles monotonic",
    ])
    assert any("remapped 1 ctaid" in n for n in notes)
    assert any("polite tier only" in n for n in notes)  # index-based stream


def test_weave_softmax_masks_score_not_values():
    out, notes = weave(fixture("softmax_decode.ll"))
    verify(out)
    check_order(out, [
        r"%s = fmul float %s\.next, %scale",
        r"%sched\.keep = icmp ult i32 %t, %sched\.budget",
        r"%sched\.shed\.score = select i1 %sched\.keep, float %s, float 0xFFF0000000000000",
        r"%m\.next = call float @llvm\.maxnum\.f32\(float %m, float %sched\.shed\.score\)",
        r"%ds = fsub float %sched\.shed\.score, %m\.next",
    ])
    assert out.count("%sched.shed.score = ") == 1
    assert "%sched.shed.val" not in out  # V loads untouched in a softmax kernel
    # the accumulator the kernel reads back and rewrites is never a stream site:
    # no L2 hint may follow its load, and no discard is ever emitted
    check_order(out, [r"%av = load float, ptr %a\.gep"])
    after = out.split("%av = load float, ptr %a.gep", 1)[1].split("\n", 2)[1]
    assert "applypriority" not in after and "discard" not in out
    assert any("softmax score mask" in n for n in notes)


@pytest.mark.parametrize("knob,absent", [
    ("SCHED_NO_INDIRECT", "%sched.task.mapped"),
    ("SCHED_NO_TIMER", "%sched.t0"),
    ("SCHED_NO_SHED", "%sched.keep"),
    ("SCHED_NO_POLICY", "applypriority.global.L2"),
])
def test_disable_knobs(knob, absent):
    out, _ = weave(fixture("paged_linear.ll"), {knob: "1"})
    verify(out)
    assert absent not in out
    full, _ = weave(fixture("paged_linear.ll"))
    assert absent in full


def test_pdl_points():
    out, _ = weave(fixture("paged_linear.ll"), {"SCHED_PDL": "1"})
    verify(out)
    check_order(out, [r"griddepcontrol\.wait", r"griddepcontrol\.launch_dependents;.*\n\s*ret void"])


@pytest.mark.parametrize("clc", [False, True])
def test_workqueue_driver(clc):
    env = {"SCHED_WORKQUEUE": "1"}
    if clc:
        env["SCHED_CLC"] = "1"
    text = fixture("paged_linear.ll")
    if not clc:
        text = text.replace("@__sched_timer = ", "@__sched_queue = addrspace(1) externally_initialized global ptr null, align 8\n@__sched_timer = ")
    out, notes = weave(text, env)
    verify(out)
    check_order(out, [
        r"define ptx_kernel void @paged_linear\(.*\"sched-wq-driver\"",
        r"%sched\.grid1d = and i1",
        r"br i1 %sched\.wq\.armed, label %sched\.dyn, label %sched\.stock",
        r"sched\.stock:",
        r"call void @paged_linear\.sched_body\(",
        r"sched\.dyn:",
        r"%sched\.ntasks = load i32",
        r"sched\.loop:",
        r"%sched\.raw = phi i32 \[ %sched\.first, %sched\.bound \], \[ %sched\.raw\.next, %sched\.claimed \]",
        r"call void @paged_linear\.sched_body\(",
        r"call void @llvm\.nvvm\.barrier0\(\)",
        r"sched\.claim:",
        (r"clusterlaunchcontrol\.try_cancel" if clc else r"atomicrmw add ptr %sched\.queue\.slot, i32 1"),
        r"sched\.claimed:",
        r"define internal void @paged_linear\.sched_body\(.*i32 %sched\.task\.arg\).*\"sched-task-body\"",
        r"%row = mul i32 %sched\.task\.arg, %nb",
        r"atomicrmw add ptr %sched\.timer\.row",
    ])
    if clc:
        assert "setp.lt.u32 %pl, %cnt" in out  # the claim's wait is bounded


def test_baked_addresses_use_a_non_constant_slot():
    text = fixture("paged_linear.ll")
    for g in ("@__sched_task_order", "@__sched_ctrl", "@__sched_timer"):
        text = "\n".join(l for l in text.splitlines() if not l.startswith(g + " ="))
    base = 0x5C00_0000_0000
    env = {"SCHED_BAKE_TASK_ORDER": base, "SCHED_BAKE_CTRL": base + 0x40000, "SCHED_BAKE_TIMER": base + 0x80000}
    out, _ = weave(text, env)
    verify(out)
    assert f"@__sched_ctrl.bakedslot = internal addrspace(1) global i64 {base + 0x40000}" in out
    assert "inttoptr i64 %sched.ctrl.baked" in out


def test_no_slots_no_weave():
    text = fixture("paged_linear.ll")
    for g in ("@__sched_task_order", "@__sched_ctrl", "@__sched_timer"):
        text = "\n".join(l for l in text.splitlines() if not l.startswith(g + " ="))
    out, _ = weave(text)
    verify(out)
    assert "%sched.task.mapped" not in out and "%sched.t0" not in out


def test_manifest_mirror_matches_cpp():
    rows = manifest_csv()
    assert [r["name"] for r in rows] == [m[0] for m in MANIFEST]
    for r, m in zip(rows, MANIFEST):
        name, effect, min_sm, knob, disables, tag = m
        assert r["effect"] == effect and int(r["minSm"]) == min_sm and r["knob"] == knob
        assert int(r["disableKnob"]) == int(disables) and r["tag"] == tag
    assert [int(r["order"]) for r in rows] == list(range(len(rows)))


def test_weave_arith_stream_prefetches_ahead():
    """Arithmetic stream (the reference's arith_decode fixture): the KV
    address is affine in the canonical IV, so the urgent tier prefetches a
    fixed distance ahead (8 iterations x 64 floats = 2048 bytes for the KV
    stream, 8 x 4 bytes for the weights), under the urgency predicate."""
    out, notes = weave(fixture("arith_decode.ll"))
    verify(out)
    check_order(out, [
        r"define ptx_kernel void @arith_decode\(",
        r"%sched\.task = select i1 %sched\.task\.ok",
        r"%sched\.pf\.ahead = add i64 %sched\.pf\.int, 2048",
        r"prefetch\.global\.L2::evict_last \[\$0\]; \}\", \"l,r,~\{memory\}\"\(i64 %sched\.pf\.ahead, i32 %sched\.urgent\.i32\)",
        r"%v = load float",
    ])
    assert "%sched.pf.ahead.1 = add i64 %sched.pf.int.1, 32" in out
    assert not any("polite tier only" in n for n in notes)


def test_arith_fixture_runs_bit_exact_on_the_host():
    """The woven arith fixture executed on the CPU (hint-only asm dropped):
    urgent policy + reversed pi leave the result bit-exact; tau truncates the
    contraction exactly."""
    import ctypes
    import struct

    import numpy as np

    from sched_pass_b200.compiler.cpu_exec import HostKernel
    from sched_pass_b200.runtime import abi

    src = fixture("arith_decode.ll")
    woven, _ = weave(src)
    stock, wk = HostKernel(src), HostKernel(woven)
    R, NT, D = 6, 40, 64
    rng = np.random.default_rng(4)
    kv = rng.standard_normal((R * NT, D)).astype(np.float32)
    w = rng.standard_normal(NT).astype(np.float32)
    p = ctypes.c_void_p

    def run(k, tables=None):
        out = np.zeros((R, D), np.float32)
        if tables is not None:
            order, ctrl = tables
            k.set_global_ptr("__sched_task_order", order.ctypes.data)
            k.set_global_ptr("__sched_ctrl", ctrl.ctypes.data)
        k.run("arith_decode", (R,), (D,), [kv.ctypes.data, w.ctypes.data, out.ctypes.data, NT],
              [p, p, p, ctypes.c_int32])
        return out

    base = run(stock)
    assert np.allclose(base, (kv.reshape(R, NT, D) * w[None, :, None]).sum(1), atol=1e-4)
    order = np.arange(R - 1, -1, -1, dtype=np.int32)
    ctrl = np.zeros(abi.ctrl_bytes(64), np.uint8)
    struct.pack_into("<I", ctrl, abi.CTRL_ORDER_SIZE_OFF, R)
    for r in range(R):
        struct.pack_into("<fHB", ctrl, abi.CTRL_ROWS_OFF + abi.ROW_SIZE * r, 1.0, 0, 1)  # urgent
    assert np.array_equal(run(wk, (order, ctrl)), base)
    tau = 13
    for r in range(R):
        struct.pack_into("<fHB", ctrl, abi.CTRL_ROWS_OFF + abi.ROW_SIZE * r, 0.0, tau, 0)
    cut = run(wk, (order, ctrl))
    want = (kv.reshape(R, NT, D)[:, :tau] * w[None, :tau, None]).sum(1)
    assert np.allclose(cut, want, atol=1e-4) and not np.allclose(cut, base, atol=1e-3)


def test_cp_async_source_warming():
    """A cp.async whose global source is affine in the canonical IV is an
    async stream site (the reference's cp.async detection): the urgent tier
    warms the source 8 iterations ahead (64 floats = 256 bytes per iteration
    -> 2048), predicated on the urgency flag and placed before the copy; the
    copy itself, its wait and the shared-memory load are untouched; the
    policy knob removes it."""
    src = fixture("async_copy.ll")
    out, notes = weave(src)
    verify(out)
    check_order(out, [
        r"%sched\.urgent = or i1",
        r"%sched\.apf\.int = ptrtoint ptr addrspace\(1\) %g to i64",
        r"%sched\.apf\.ahead = add i64 %sched\.apf\.int, 2048",
        r"prefetch\.global\.L2::evict_last \[\$0\]; \}\", \"l,r,~\{memory\}\"\(i64 %sched\.apf\.ahead, i32 %sched\.urgent\.i32\)",
        r"call void asm sideeffect \"cp\.async\.ca\.shared\.global \[\$0\], \[\$1\], 4;\"",
        r"cp\.async\.wait_all",
        r"%v = load float, ptr addrspace\(3\) %sh",
    ])
    assert any("cp.async source warming woven" in n for n in notes)
    assert "%sched.keep" not in out  # shared-memory data: no value mask
    off, _ = weave(src, {"SCHED_NO_POLICY": "1"})
    assert "%sched.apf" not in off


def test_tma_stream_warming():
    """A tiled TMA load (cp.async.bulk.tensor, global -> shared) whose box
    coordinate is affine in the canonical IV is a TMA stream site: the urgent
    tier prefetches the box 8 iterations ahead (innermost coordinate +64 per
    iteration -> +512, the row coordinate unchanged) with
    cp.async.bulk.prefetch.tensor right before the load, which itself stays
    untouched; the policy knob removes it. The woven module assembles for
    sm_100a (ptxas is given the generated PTX and only its status is used)."""
    import shutil
    import subprocess
    import tempfile
    src = fixture("tma_stream.ll")
    out, notes = weave(src)
    verify(out)
    check_order(out, [
        r"%sched\.urgent = or i1",
        r"%sched\.tpf\.c = add i32 %x, 512",
        r"@p cp\.async\.bulk\.prefetch\.tensor\.2d\.L2\.global\.tile \[\$0, \{\$1, \$2\}\]; \}\", \"l,r,r,r,~\{memory\}\"\(ptr %tmap, i32 %sched\.tpf\.c, i32 %y, i32 %sched\.urgent\.i32\)",
        r"@p cp\.async\.bulk\.tensor\.2d\.shared::cluster\.global\.tile\.mbarrier::complete_tx::bytes \[\$0\], \[\$1, \{\$2, \$3\}\], \[\$4\]",
        r"mbarrier\.try_wait\.parity",
        r"%v = load i16, ptr addrspace\(3\) %sh",
    ])
    assert any("TMA stream warming woven" in n for n in notes)
    assert "%sched.keep" not in out  # shared-memory data: no value mask
    off, _ = weave(src, {"SCHED_NO_POLICY": "1"})
    assert "%sched.tpf" not in off and "prefetch.tensor" not in off
    ptxas = shutil.which("ptxas") or "/usr/local/cuda/bin/ptxas"
    if not os.path.exists(ptxas):
        pytest.skip("ptxas not installed")
    from sched_pass_b200.compiler.nvptx import compile_ptx
    with tempfile.TemporaryDirectory() as d:
        ptx = os.path.join(d, "k.ptx")
        with open(ptx, "wb") as fh:
            fh.write(compile_ptx(out))
        r = subprocess.run([ptxas, "-arch=sm_100a", ptx, "-o", os.path.join(d, "k.cubin")],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-2000:]


def test_tma_parser_declines_stores_and_fixed_boxes():
    """Stores (global before shared), im2col boxes and prefetches are not
    stream loads; a load whose coordinates never move with the loop is
    declined with a note."""
    src = fixture("tma_stream.ll")
    store = src.replace("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [$0], [$1, {$2, $3}], [$4]",
                        "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [$1, {$2, $3}], [$0]")
    out, notes = weave(store)
    assert "%sched.tpf" not in out and not any("TMA stream" in n for n in notes)
    fixed = src.replace("%x = mul i32 %k, 64", "%x = mul i32 %req, 64")
    out, notes = weave(fixed)
    assert "%sched.tpf" not in out
    assert any("no coordinate advances with the loop" in n for n in notes)


def test_manifest_markdown_lists_every_lever_in_order():
    from sched_pass_b200.runtime.manifest import manifest_markdown
    rows = manifest_markdown().splitlines()[2:]
    assert [r.split("|")[2].strip() for r in rows] == [m[0] for m in MANIFEST]
    assert "`SCHED_NO_SHED`" in rows[2] and "`-nos`" in rows[2]


def test_command_line_weave_and_manifest(tmp_path):
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(HERE))
    out = tmp_path / "w.ll"
    r = subprocess.run([sys.executable, "-m", "sched_pass_b200", "weave", os.path.join(HERE, "paged_linear.ll"),
                        "-o", str(out), "--env", "SCHED_PDL=1"], capture_output=True, text=True, cwd=root)
    assert r.returncode == 0, r.stderr
    text = out.read_text()
    verify(text)
    assert "griddepcontrol.wait" in text and "remapped 1 ctaid" in r.stderr
    m = subprocess.run([sys.executable, "-m", "sched_pass_b200", "manifest", "--csv"], capture_output=True,
                       text=True, cwd=root)
    assert m.returncode == 0 and m.stdout.splitlines()[0] == "name,effect,minSm,knob,disableKnob,order,tag"


def test_doctor_reports_the_environment():
    from sched_pass_b200.__main__ import doctor
    rep = doctor()
    for k in ("python", "torch", "gpus", "peer_access", "nccl", "nvcc", "native", "measured_peaks"):
        assert k in rep
    assert set(rep["native"]) == {"extension", "weaver", "host_runtime"}


def test_loops_come_from_dominators_not_block_order():
    """A loop whose latch precedes its header in the text, whose body spans
    two blocks around the exit block, and whose IV phi lists the back edge
    first (``add nuw nsw i32 1, %i``): the weaver finds it through the
    dominator tree, weaves shed on its canonical IV, and the woven kernel run
    on the host is bit-exact with null slots and exactly truncated with a
    tau budget."""
    import ctypes
    import struct

    import numpy as np

    from sched_pass_b200.compiler.cpu_exec import HostKernel
    from sched_pass_b200.runtime import abi

    src = fixture("paged_linear_shuffled.ll")
    woven, notes = weave(src)
    verify(woven)
    text = "\n".join(notes) if isinstance(notes, (list, tuple)) else str(notes)
    assert "no canonical induction variable" not in text, text
    assert "shed linear value mask woven" in text, text
    assert "%sched.keep" in woven and "icmp ult i32 %i," in woven
    R, NB, D = 5, 9, 64
    rng = np.random.default_rng(5)
    kv = rng.standard_normal((R * NB, 64)).astype(np.float32)
    bt = rng.permutation(R * NB).astype(np.int32)
    w = rng.standard_normal(NB).astype(np.float32)
    p = ctypes.c_void_p

    def run(k, tables=None):
        out = np.zeros((R, D), np.float32)
        if tables is not None:
            order, ctrl = tables
            k.set_global_ptr("__sched_task_order", order.ctypes.data)
            k.set_global_ptr("__sched_ctrl", ctrl.ctypes.data)
        k.run("paged_linear_shuffled", (R,), (D,), [kv.ctypes.data, bt.ctypes.data, w.ctypes.data, out.ctypes.data,
                                                     NB], [p, p, p, p, ctypes.c_int32])
        return out

    stock = run(HostKernel(src))
    want = np.stack([(kv[bt[r * NB:(r + 1) * NB]] * w[:, None]).sum(0) for r in range(R)])
    assert np.allclose(stock, want, atol=1e-4)
    wk = HostKernel(woven)
    assert np.array_equal(run(wk), stock)  # null slots: bit-exact
    order = np.arange(R - 1, -1, -1, dtype=np.int32)
    ctrl = np.zeros(abi.ctrl_bytes(64), np.uint8)
    struct.pack_into("<I", ctrl, abi.CTRL_ORDER_SIZE_OFF, R)
    assert np.array_equal(run(wk, (order, ctrl)), stock)  # reversed order, no budget: still exact
    tau = 4
    for r in range(R):
        struct.pack_into("<fHB", ctrl, abi.CTRL_ROWS_OFF + abi.ROW_SIZE * r, 0.0, tau, 0)
    cut = run(wk, (order, ctrl))
    want_cut = np.stack([(kv[bt[r * NB:r * NB + tau]] * w[:tau, None]).sum(0) for r in range(R)])
    assert np.allclose(cut, want_cut, atol=1e-4) and not np.allclose(cut, stock, atol=1e-3)
