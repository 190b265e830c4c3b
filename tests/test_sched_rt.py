"""The fixed-VA control arena and its failure modes, on the CPU (the arena
is mapped without registering it with CUDA). Each test runs in a child
process: the arena is one per process."""
import ctypes
import os
import struct
import subprocess
import sys
import textwrap

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_child(body: str) -> str:
    code = "import sys; sys.path.insert(0, %r)\n" % ROOT + textwrap.dedent(body)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120,
                       env={**os.environ, "CUDA_VISIBLE_DEVICES": ""})
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout + r.stderr


def test_arena_layout_push_order_and_rows():
    out = run_child("""
        import struct, torch, numpy as np
        from sched_pass_b200.runtime.sched_rt import SchedPlane
        from sched_pass_b200.runtime import abi
        p = SchedPlane(max_tasks=64, device="cpu", mode="arena")
        a = p.arena
        assert a.canonical and a.base == abi.DEFAULT_VA_BASE
        p.install_order(torch.arange(63, -1, -1), 64)
        p.set_num_tasks(64); p.set_timer_enabled(False)
        p.set_rows(q=np.linspace(0, 1, 64, dtype=np.float32), tau=np.arange(64), hint=np.full(64, 2))
        p.push()
        ctrl = a.read(abi.CTRL_OFF, abi.ctrl_bytes(64))
        gen, ntask = struct.unpack_from("<II", ctrl, 0)
        flags, osize = struct.unpack_from("<II", ctrl, abi.CTRL_FLAGS_OFF)
        q, tau, hint = struct.unpack_from("<fHB", ctrl, abi.CTRL_ROWS_OFF + abi.ROW_SIZE * 10)
        order = np.frombuffer(a.read(abi.ORDER_OFF, 4 * 64), dtype=np.int32)
        assert gen == p.generation and ntask == 64 and osize == 64 and flags & abi.FLAG_TIMER_OFF
        assert abs(q - 10 / 63) < 1e-6 and tau == 10 and hint == 2
        assert order[0] == 63 and order[-1] == 0
        p.set_row(10, q=0.5, tau=7, hint=1); p.push()
        q, tau, hint = struct.unpack_from("<fHB", a.read(abi.CTRL_OFF, abi.ctrl_bytes(64)), abi.CTRL_ROWS_OFF + abi.ROW_SIZE * 10)
        assert (q, tau, hint) == (0.5, 7, 1)
        print("OK")
    """)
    assert "OK" in out


def test_canonical_va_miss_relocates_and_rekeys_the_cache():
    out = run_child("""
        import ctypes
        from sched_pass_b200.runtime.sched_rt import SchedPlane, compute_bake_env
        from sched_pass_b200.runtime import abi
        libc = ctypes.CDLL(None)
        libc.mmap.restype = ctypes.c_void_p
        libc.mmap.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_long]
        blocker = libc.mmap(ctypes.c_void_p(abi.DEFAULT_VA_BASE), abi.ARENA_BYTES, 3, 0x22 | 0x100000, -1, 0)
        assert blocker == abi.DEFAULT_VA_BASE, hex(blocker or 0)
        p = SchedPlane(max_tasks=64, device="cpu", mode="arena")
        assert not p.arena.canonical and p.arena.base != abi.DEFAULT_VA_BASE
        env = p.bake_env("/bin/true")
        assert f"va{p.arena.base:x}" in env["SCHED_KERNEL_CACHE"]
        assert int(env["SCHED_BAKE_CTRL"]) == p.arena.base + abi.CTRL_OFF
        canon = compute_bake_env(abi.DEFAULT_VA_BASE, 64, "/bin/true", {})
        assert canon["SCHED_KERNEL_CACHE"] != env["SCHED_KERNEL_CACHE"]
        print("OK")
    """)
    assert "OK" in out and "canonical VA" in out  # the relocation is announced


def test_oversized_batch_and_corrupted_order_are_refused():
    out = run_child("""
        import torch
        from sched_pass_b200.runtime.sched_rt import SchedPlane
        p = SchedPlane(max_tasks=32, device="cpu", mode="arena")
        try:
            p.install_order(torch.arange(40), 40)
            raise SystemExit("oversized batch accepted")
        except RuntimeError as e:
            assert "SCHED_MAX_TASKS" in str(e)
        bad = torch.tensor([0, 1, 1, 3])
        try:
            p.install_order(bad, 4)
            raise SystemExit("duplicate-entry order accepted")
        except ValueError:
            pass
        try:
            p.install_order(torch.tensor([0, 1, 2, 9]), 4)
            raise SystemExit("out-of-range order accepted")
        except ValueError:
            pass
        p.install_order(torch.tensor([3, 2, 1, 0]), 4)
        print("OK")
    """)
    assert "OK" in out


def test_second_arena_in_one_process_is_refused():
    out = run_child("""
        from sched_pass_b200.runtime.sched_rt import SchedArena, SchedArenaError
        a = SchedArena(cuda=False)
        try:
            SchedArena(cuda=False)
            raise SystemExit("second arena accepted")
        except SchedArenaError:
            pass
        a.close()
        b = SchedArena(cuda=False)  # after close, a new one may be made
        b.close()
        print("OK")
    """)
    assert "OK" in out


PHASE = """
    import json, os, sys
    import numpy as np, torch
    sys.path.insert(0, os.path.join(%(root)r, "tests"))
    from test_config0_cpu import B, build, reference, run
    from sched_pass_b200.compiler.cpu_exec import HostKernel
    from sched_pass_b200.compiler.weave import weave_cached, weaver_path
    from sched_pass_b200.runtime.sched_rt import SchedPlane, compute_bake_env
    p = SchedPlane(max_tasks=64, device="cpu", mode="arena")
    assert p.arena.canonical
    env = compute_bake_env(p.arena.base, 64, weaver_path(), {"SCHED_CACHE_ROOT": %(cache)r})
    src = open(os.path.join(%(root)r, "tests", "ir", "softmax_decode.ll")).read()
    src = "\\n".join(l for l in src.splitlines() if not l.startswith("@__sched_"))  # baked ABI: no named slots
    woven, notes, hit = weave_cached(src, env, "softmax_decode")
    k = HostKernel(woven)
    lens, bt, kc, vc, q, taus, maxp = build(5)
    p.install_order(torch.arange(B - 1, -1, -1), B)
    p.set_num_tasks(B)
    p.set_rows(tau=taus.astype(np.int64), n=B)
    p.push()
    out = run(k, lens, bt, kc, vc, q, maxp)  # tables reached through the baked arena addresses
    err = float(np.abs(out - reference(lens, bt, kc, vc, q, taus)).max())
    timer = p.read_timer()[:B]
    print("PHASE " + json.dumps({"hit": hit, "base": p.arena.base, "err": err,
                                 "timer_rows": int((timer > 0).sum()), "cache": env["SCHED_KERNEL_CACHE"]}))
"""


def test_two_processes_share_the_arena_va_and_the_woven_kernel(tmp_path):
    """The reference's fixed-VA check (test/py/test_fixed_va.py): two
    processes in turn map the arena at the canonical VA, derive the same
    cache key, and the second reuses the first one's woven module, whose
    baked table addresses then reach the second process's arena (reversed
    pi + per-request tau: exact truncated attention, timer rows filled)."""
    import json
    res = []
    for _ in range(2):
        out = run_child(PHASE % {"root": ROOT, "cache": str(tmp_path)})
        line = [l for l in out.splitlines() if l.startswith("PHASE ")]
        assert line, out
        res.append(json.loads(line[0][len("PHASE "):]))
    assert [r["hit"] for r in res] == [False, True], res
    assert res[0]["base"] == res[1]["base"] and res[0]["cache"] == res[1]["cache"]
    for r in res:
        assert r["err"] < 1e-4 and r["timer_rows"] == 8, r
