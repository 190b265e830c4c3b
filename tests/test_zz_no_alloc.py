"""The fixed-scratch GEMM entry point, called through its exported C symbol.

``sched_gemm_run_fixed_scratch`` runs the stream-K tcgen05 GEMM with scratch
that lives in the module's own device arrays, so the call allocates nothing
(for callers that may not allocate device memory). It is checked bit for bit
against the regular entry point (``ops.linear``, which hands the kernel a
caller-owned workspace) with the same explicit grid, on shapes whose tiles
are split across CTAs under that grid, i.e. calls that really use the
scratch, twice in a row each: the second call only agrees if the first left
the tile counters at zero. Both entry points run the same deterministic
schedule, so the outputs must be equal. This file is named to be collected
last so that it also runs after every other GPU test.
"""
import ctypes
import math

import pytest
import torch

from sched_pass_b200 import _build, ops
from sched_pass_b200._ext import ext

pytestmark = pytest.mark.gpu

EPI_STORE, EPI_SWIGLU, EPI_ALLREDUCE = 0, 1, 3
TOO_LARGE, BAD_EPILOGUE = -8, -10
WS_CAP = 1 << 22


class GemmArgs(ctypes.Structure):
    """Mirror of the C struct GemmArgs (natural x86-64 layout)."""
    _fields_ = [
        ("x", ctypes.c_void_p), ("ldx", ctypes.c_int),
        ("w", ctypes.c_void_p), ("y", ctypes.c_void_p), ("ldy", ctypes.c_int),
        ("T", ctypes.c_int), ("N", ctypes.c_int), ("K", ctypes.c_int),
        ("epi", ctypes.c_int), ("grid", ctypes.c_int), ("num_sms", ctypes.c_int),
        ("ws", ctypes.c_void_p), ("ws_floats", ctypes.c_longlong),
        ("counters", ctypes.c_void_p), ("counter_count", ctypes.c_int),
        ("status", ctypes.c_void_p),
        ("pos", ctypes.c_void_p), ("slot", ctypes.c_void_p), ("cos_sin", ctypes.c_void_p),
        ("q_out", ctypes.c_void_p), ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
        ("Hq", ctypes.c_int), ("Hkv", ctypes.c_int), ("page_size", ctypes.c_int),
        ("rank", ctypes.c_int), ("world", ctypes.c_int),
        ("recv", ctypes.c_void_p * 8), ("flags", ctypes.c_void_p * 8),
        ("trace", ctypes.c_void_p), ("kv_pages", ctypes.c_int),
        ("x_ready", ctypes.c_void_p),
        ("ll_state", ctypes.c_void_p), ("ll_set_lines", ctypes.c_longlong),
        ("norm_res", ctypes.c_void_p), ("norm_w", ctypes.c_void_p), ("norm_out", ctypes.c_void_p),
        ("row_cnt", ctypes.c_void_p), ("norm_eps", ctypes.c_float),
        ("ll_mc", ctypes.c_void_p),
    ]


@pytest.fixture(scope="module")
def lib():
    ext()  # builds / loads the extension; ctypes then shares the loaded image
    so = ctypes.CDLL(_build.ext_path())
    so.sched_gemm_run_fixed_scratch.argtypes = [ctypes.POINTER(GemmArgs), ctypes.c_void_p]
    so.sched_gemm_run_fixed_scratch.restype = ctypes.c_int
    so.sched_gemm_ws_floats.argtypes = [ctypes.c_int] * 4
    so.sched_gemm_ws_floats.restype = ctypes.c_longlong
    so.sched_gemm_plan.argtypes = [ctypes.c_int] * 5 + [ctypes.POINTER(ctypes.c_int)] * 2
    so.sched_gemm_plan.restype = None
    so.sched_gemm_fixed_scratch_reset.argtypes = [ctypes.c_void_p]
    so.sched_gemm_fixed_scratch_reset.restype = ctypes.c_int
    return so


def default_plan(lib, T, N, K, epi):
    cs, grid = ctypes.c_int(), ctypes.c_int()
    lib.sched_gemm_plan(T, N, K, epi, torch.cuda.get_device_properties(0).multi_processor_count,
                        ctypes.byref(cs), ctypes.byref(grid))
    return cs.value, grid.value


def call(lib, x, w, y, epi, grid):
    st = ops.status_buffer(x.device)
    a = GemmArgs(x=x.data_ptr(), ldx=x.stride(0), w=w.data_ptr(), y=y.data_ptr(), ldy=y.stride(0),
                 T=x.shape[0], N=w.shape[0], K=x.shape[1], epi=epi, grid=grid,
                 num_sms=torch.cuda.get_device_properties(x.device).multi_processor_count,
                 status=st.data_ptr())
    return lib.sched_gemm_run_fixed_scratch(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("T,N,K,epi,grid", [
    (1, 4096, 4096, EPI_STORE, 148),
    (16, 6144, 4096, EPI_STORE, 148),
    (40, 4096, 1024, EPI_STORE, 97),
    (16, 4096, 2048, EPI_SWIGLU, 120),
    (64, 2048, 4096, EPI_SWIGLU, 148),
])
def test_fixed_scratch_matches_regular_entry_point(lib, T, N, K, epi, grid):
    # an explicit grid always runs stream-K; these shapes split tiles under it
    assert lib.sched_gemm_ws_floats(T, N, K, grid) > 0, "shape must split tiles (use the scratch)"
    g = torch.Generator(device="cuda").manual_seed(T * 7 + N)
    x = torch.randn(T, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).to(torch.bfloat16)
    cols = N // 2 if epi == EPI_SWIGLU else N
    want = ops.linear(x, w, swiglu=epi == EPI_SWIGLU, grid=grid)
    for _ in range(2):
        y = torch.full((T, cols), float("nan"), dtype=torch.bfloat16, device="cuda")
        assert call(lib, x, w, y, epi, grid) == 0
        torch.cuda.synchronize()
        ops.check_status()
        assert torch.equal(y, want)


def test_default_grid_cluster_schedule_is_not_refused(lib):
    """A default-grid call that the planner runs as cluster split-K needs no
    scratch: it runs (and matches the regular entry point) even when its
    stream-K plan would need more scratch than the fixed capacity."""
    shapes = [(T, N, K) for T in (1, 16) for N, K in ((4096, 4096), (4096, 14336))]
    cluster = [(T, N, K) for T, N, K in shapes if default_plan(lib, T, N, K, EPI_STORE)[0] > 0]
    if not cluster:
        pytest.skip("no decode shape plans as cluster split-K on this GPU")
    for T, N, K in cluster:
        x = torch.randn(T, K, device="cuda").to(torch.bfloat16)
        w = (torch.randn(N, K, device="cuda") / math.sqrt(K)).to(torch.bfloat16)
        want = ops.linear(x, w, grid=0)
        y = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
        assert call(lib, x, w, y, EPI_STORE, 0) == 0
        torch.cuda.synchronize()
        ops.check_status()
        assert torch.equal(y, want)


def test_fixed_scratch_refuses_what_it_cannot_hold(lib):
    T, N, K = 256, 8192, 4096
    assert lib.sched_gemm_ws_floats(T, N, K, 148) > WS_CAP
    x = torch.zeros(T, K, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(N, K, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros(T, N, dtype=torch.bfloat16, device="cuda")
    assert call(lib, x, w, y, EPI_STORE, 148) == TOO_LARGE
    assert call(lib, x, w, y, EPI_ALLREDUCE, 148) == BAD_EPILOGUE
    torch.cuda.synchronize()
    ops.check_status()
    # the reset (for after a call that reported a status) zeroes the counters
    # with a memset on the stream; calls after it still agree bit for bit
    assert lib.sched_gemm_fixed_scratch_reset(torch.cuda.current_stream().cuda_stream) == 0
    xs = torch.randn(16, 4096, device="cuda").to(torch.bfloat16)
    ws = (torch.randn(6144, 4096, device="cuda") / 64).to(torch.bfloat16)
    ys = torch.empty(16, 6144, dtype=torch.bfloat16, device="cuda")
    assert call(lib, xs, ws, ys, EPI_STORE, 148) == 0
    torch.cuda.synchronize()
    ops.check_status()
    assert torch.equal(ys, ops.linear(xs, ws, grid=148))


def test_default_grid_pair_schedule_uses_the_fixed_scratch(lib, monkeypatch):
    """A default-grid prefill-size call runs the CTA-pair kernel, whose last
    wave's k-range partials fit the fixed scratch here (T=512: 32 tiles, 2
    k-ranges each, exactly its capacity): not refused, and bit-identical to
    the regular entry point, which plans the same schedule, on two calls in a
    row (the second agrees only if the first left its counters at zero)."""
    monkeypatch.delenv("SCHED_GEMM_PAIR", raising=False)
    monkeypatch.delenv("SCHED_GEMM_PAIR_SPLIT", raising=False)
    T, N, K = 512, 4096, 4096
    np_, _, splits = ext().gemm_pair_plan(T, N, K, EPI_STORE, WS_CAP, 1 << 14)
    if np_ == 0:
        pytest.skip("the pair schedule is not planned for this shape on this GPU")
    assert splits > 1
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(T, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).to(torch.bfloat16)
    want = ops.linear(x, w)
    for _ in range(2):
        y = torch.full((T, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        assert call(lib, x, w, y, EPI_STORE, 0) == 0
        torch.cuda.synchronize()
        ops.check_status()
        assert torch.equal(y, want)
