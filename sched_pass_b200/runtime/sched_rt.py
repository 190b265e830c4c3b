"""The Python control plane: control tables, their addresses, per-step writes.

API-compatible with the reference plane (python/sched_rt.py:186-609 of
jc-su/sched-pass): ``SchedPlane`` keeps its constructor and its setters
(``set_order``, ``install_order``, ``set_row(s)``, ``set_num_tasks``,
``set_timer_enabled``, ``push``, ``read_timer``, ``clear_timer``,
``reset_queue``, ``region_order``...), and ``SchedArena`` keeps the fixed
virtual-address arena that lets a kernel compiled with baked table addresses
stay valid in a later process.

Two table homes, one setter API:

* ``mode="arena"`` (the reference's baked ABI): all tables in one host
  mapping at a canonical VA (``mmap(MAP_FIXED_NOREPLACE)``), registered with
  CUDA so the device pointer equals the host pointer. Publishing is a plain
  memcpy; kernels read the tables over PCIe. ``use_device_timer`` /
  ``use_device_order`` turn the timer / order words into pointers to device
  tensors (the "indirect" channels).
* ``mode="device"`` (this framework's default for serving): order, control
  block, timer and ticket queue live in device memory; a pinned host mirror is
  published with one stream-ordered copy (body first, generation word last),
  so a serving loop never synchronises and the copy can sit in front of a
  CUDA-graph replay. Device atomics replace the PCIe timer atomics.

The kernels of this framework take the tables as a by-value ``SchedSlots``
launch argument: ``plane.slots()`` returns the tensors/pointers for it.
"""
from __future__ import annotations

import atexit
import ctypes
import hashlib
import os
import struct

import torch

from . import abi
from .abi import (ARENA_BYTES, CTRL_FLAGS_OFF, CTRL_LAMBDA_OFF, CTRL_NUM_TASKS_OFF,
                  CTRL_OFF, CTRL_ORDER_SIZE_OFF, CTRL_ROWS_OFF, DEFAULT_VA_BASE,
                  FLAG_TIMER_OFF, HINT_AUTO, HINT_POLITE, HINT_URGENT, MAX_TASKS_LIMIT,
                  ORDER_OFF, QUEUE_OFF, ROW_SIZE, TIMER_OFF)
from .manifest import MANIFEST, disable_mask

__all__ = [
    "SchedArena", "SchedArenaError", "SchedPlane", "compute_bake_env", "predicted_base",
    "HINT_AUTO", "HINT_URGENT", "HINT_POLITE", "MANIFEST",
]

_MAP_FIXED_NOREPLACE = 0x100000
_MAP_ANON_PRIVATE = 0x22
_PROT_RW = 0x3
_CU_MEMHOSTREGISTER_DEVICEMAP = 0x02


class SchedArenaError(RuntimeError):
    """An OS or CUDA call underneath the arena failed."""


def predicted_base() -> int:
    """The VA the arena will ask for: ``SCHED_VA_BASE`` or the default."""
    return int(os.environ.get("SCHED_VA_BASE", "0"), 0) or DEFAULT_VA_BASE


def _file_tag(path: str) -> str:
    try:
        h = hashlib.sha256()
        with open(path, "rb") as f:
            for chunk in iter(lambda: f.read(1 << 20), b""):
                h.update(chunk)
        return h.hexdigest()[:8]
    except OSError:
        return "none"


def compute_bake_env(base: int, max_tasks: int, weaver: str, base_env,
                     timer_indirect: bool = False, order_indirect: bool = False) -> dict:
    """Environment of a weave that bakes the arena at ``base`` into the code.

    Pure function of its inputs, so a JIT cache directory can be chosen before
    the arena exists. The cache key holds every weave input that changes the
    generated code: base VA, table capacity, acquisition mode, indirect
    channels, the lever-disable mask (derived from the manifest) and a hash of
    the weaver binary. Variable names of the reference's bake protocol are
    kept (SCHED_BAKE_*, SCHED_MAX_TASKS, SCHED_*_INDIRECT).
    """
    env = dict(base_env)
    env["SCHED_WEAVER"] = weaver
    env["SCHED_BAKE_TASK_ORDER"] = str(base + ORDER_OFF)
    env["SCHED_BAKE_CTRL"] = str(base + CTRL_OFF)
    env["SCHED_BAKE_TIMER"] = str(base + TIMER_OFF)
    env["SCHED_BAKE_QUEUE"] = str(base + QUEUE_OFF)
    env["SCHED_MAX_TASKS"] = str(max_tasks)
    if timer_indirect:
        env["SCHED_TIMER_INDIRECT"] = "1"
    if order_indirect:
        env["SCHED_ORDER_INDIRECT"] = "1"
    root = env.get("SCHED_CACHE_ROOT", os.path.join(os.path.dirname(__file__), "..", "_build", "kcache"))
    mode = ""
    if env.get("SCHED_WORKQUEUE"):
        mode = "-wqclc" if env.get("SCHED_CLC") else "-wqtk"
    if timer_indirect or env.get("SCHED_TIMER_INDIRECT"):
        mode += "-ti"
    if order_indirect or env.get("SCHED_ORDER_INDIRECT"):
        mode += "-oi"
    mask = disable_mask(env)
    if mask:
        mode += f"-no{mask}"
    mode += f"-w{_file_tag(weaver)}"
    env["SCHED_KERNEL_CACHE"] = os.path.abspath(os.path.join(root, f"va{base:x}-n{max_tasks}{mode}"))
    return env


class _PinnedRing:
    """A few pinned staging buffers for asynchronous host-to-device publishes.
    A buffer is rewritten only after the copy that last read it has executed
    (an event per buffer), so a publish never races an in-flight copy."""

    def __init__(self, nbytes: int, pinned: bool, depth: int = 4):
        self.bufs = [torch.zeros(nbytes, dtype=torch.uint8, pin_memory=pinned) for _ in range(depth)]
        self.events = [None] * depth
        self.pinned = pinned
        self.i = 0

    def stage(self, data) -> torch.Tensor:
        self.i = (self.i + 1) % len(self.bufs)
        ev = self.events[self.i]
        if ev is not None:
            ev.synchronize()
        buf = self.bufs[self.i]
        mv = memoryview(data).cast("B")
        buf[:len(mv)].numpy()[:] = np_frombuffer(mv)
        return buf

    def mark(self) -> None:
        if self.pinned:
            ev = torch.cuda.Event()
            ev.record()
            self.events[self.i] = ev


def np_frombuffer(mv):
    import numpy as np
    return np.frombuffer(mv, dtype=np.uint8)


class SchedArena:
    """The tables in one host mapping at a fixed VA, device-visible through
    ``cuMemHostRegister(DEVICEMAP)`` (under unified addressing the device
    pointer equals the host pointer). One arena per process.

    ``cuda=False`` maps the arena without registering it: tables usable by
    host-side observers and by tests on machines without a GPU.
    """

    _instance: "SchedArena | None" = None

    def __init__(self, device_ordinal: int = 0, va_base: int | None = None, cuda: bool = True):
        if SchedArena._instance is not None:
            raise SchedArenaError("SchedArena already exists in this process; reuse its SchedPlane")
        env_base = int(os.environ.get("SCHED_VA_BASE", "0"), 0)
        requested = env_base or (va_base if va_base is not None else DEFAULT_VA_BASE)
        self.size = ARENA_BYTES
        libc = ctypes.CDLL(None, use_errno=True)
        libc.mmap.restype = ctypes.c_void_p
        libc.mmap.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int,
                              ctypes.c_int, ctypes.c_long]
        libc.munmap.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
        self._libc = libc
        failed = ctypes.c_void_p(-1).value
        addr = libc.mmap(ctypes.c_void_p(requested), self.size, _PROT_RW,
                         _MAP_ANON_PRIVATE | _MAP_FIXED_NOREPLACE, -1, 0)
        if addr in (None, failed) or addr != requested:
            if addr not in (None, failed):
                libc.munmap(ctypes.c_void_p(addr), self.size)
            addr = libc.mmap(None, self.size, _PROT_RW, _MAP_ANON_PRIVATE, -1, 0)
            if addr in (None, failed):
                raise SchedArenaError("mmap of the control arena failed")
            print(f"[sched] canonical VA 0x{requested:x} is taken; arena at 0x{addr:x} "
                  f"(baked kernels for this base compile into their own cache)")
        self.base: int = addr
        self.canonical: bool = addr == requested
        self.cu = None
        self.registered = False
        if cuda:
            try:
                self.cu = ctypes.CDLL("libcuda.so.1")
            except OSError as e:
                libc.munmap(ctypes.c_void_p(self.base), self.size)
                raise SchedArenaError(f"libcuda unavailable: {e}") from e
            try:
                self._check("cuInit", self.cu.cuInit(0))
                self._ensure_context(device_ordinal)
                self._check("cuMemHostRegister", self.cu.cuMemHostRegister_v2(
                    ctypes.c_void_p(self.base), ctypes.c_size_t(self.size),
                    ctypes.c_uint(_CU_MEMHOSTREGISTER_DEVICEMAP)))
                self.registered = True
                dptr = ctypes.c_uint64()
                self._check("cuMemHostGetDevicePointer", self.cu.cuMemHostGetDevicePointer_v2(
                    ctypes.byref(dptr), ctypes.c_void_p(self.base), 0))
                if dptr.value != self.base:
                    raise SchedArenaError(
                        f"device pointer 0x{dptr.value:x} != host pointer 0x{self.base:x}: "
                        "baked addresses would be wrong")
            except Exception:
                self.close(force=True)
                raise
        ctypes.memset(ctypes.c_void_p(self.base), 0, self.size)
        SchedArena._instance = self
        atexit.register(self.close)

    def _check(self, name: str, rc: int) -> None:
        if rc != 0:
            msg = ctypes.c_char_p()
            self.cu.cuGetErrorName(rc, ctypes.byref(msg))
            raise SchedArenaError(f"{name} failed: {msg.value.decode() if msg.value else rc}")

    def _ensure_context(self, device_ordinal: int) -> None:
        ctx = ctypes.c_void_p()
        self._check("cuCtxGetCurrent", self.cu.cuCtxGetCurrent(ctypes.byref(ctx)))
        if ctx.value:
            return
        dev = ctypes.c_int()
        self._check("cuDeviceGet", self.cu.cuDeviceGet(ctypes.byref(dev), device_ordinal))
        pctx = ctypes.c_void_p()
        self._check("cuDevicePrimaryCtxRetain", self.cu.cuDevicePrimaryCtxRetain(ctypes.byref(pctx), dev))
        self._check("cuCtxSetCurrent", self.cu.cuCtxSetCurrent(pctx))

    def write(self, offset: int, data: bytes) -> None:
        if offset < 0 or offset + len(data) > self.size:
            raise ValueError("arena write out of range")
        ctypes.memmove(ctypes.c_void_p(self.base + offset), data, len(data))

    def read(self, offset: int, nbytes: int) -> bytes:
        if offset < 0 or offset + nbytes > self.size:
            raise ValueError("arena read out of range")
        return ctypes.string_at(ctypes.c_void_p(self.base + offset), nbytes)

    def memset(self, offset: int, value: int, nbytes: int) -> None:
        ctypes.memset(ctypes.c_void_p(self.base + offset), value, nbytes)

    def close(self, force: bool = False) -> None:
        if self.base and (SchedArena._instance is self or force):
            if self.registered:
                self.cu.cuMemHostUnregister(ctypes.c_void_p(self.base))
                self.registered = False
            self._libc.munmap(ctypes.c_void_p(self.base), ctypes.c_size_t(self.size))
            self.base = 0
            if SchedArena._instance is self:
                SchedArena._instance = None


class SchedPlane:
    """Per-step scheduling control plane (see the module docstring)."""

    BAKE_KEYS = ("SCHED_WEAVER", "SCHED_BAKE_TASK_ORDER", "SCHED_BAKE_CTRL", "SCHED_BAKE_TIMER",
                 "SCHED_BAKE_QUEUE", "SCHED_MAX_TASKS", "SCHED_KERNEL_CACHE",
                 "SCHED_TIMER_INDIRECT", "SCHED_ORDER_INDIRECT")

    def __init__(self, max_tasks: int = abi.DEFAULT_MAX_TASKS, device: str = "cuda",
                 va_base: int | None = None, mode: str = "arena"):
        if mode not in ("arena", "device"):
            raise ValueError("mode must be 'arena' or 'device'")
        if mode == "arena" and max_tasks > MAX_TASKS_LIMIT:
            raise ValueError(f"max_tasks {max_tasks} > {MAX_TASKS_LIMIT} (the arena's table window)")
        self.N = int(max_tasks)
        self.dev = device
        self.mode = mode
        self.ctrl_bytes = abi.ctrl_bytes(self.N)
        self._ctrl_host = bytearray(self.ctrl_bytes)
        self._generation = 0
        self._timer_dev = None
        self._order_dev = None
        self._timer_stream = None
        self.arena = None
        on_cuda = device.startswith("cuda")
        if mode == "arena":
            ordinal = 0
            if on_cuda:
                torch.cuda.init()
                ordinal = torch.cuda.current_device()
            self.arena = SchedArena(device_ordinal=ordinal, va_base=va_base, cuda=on_cuda)
        else:
            # device-resident tables + pinned mirrors
            pin = on_cuda
            self.order_t = torch.arange(self.N, dtype=torch.int32, device=device)
            self.ctrl_t = torch.zeros(self.ctrl_bytes, dtype=torch.uint8, device=device)
            self.timer_t = torch.zeros(self.N, dtype=torch.int64, device=device)
            self.queue_t = torch.zeros(4, dtype=torch.int32, device=device)
            self._ctrl_ring = _PinnedRing(self.ctrl_bytes, pin)
            self._order_ring = _PinnedRing(4 * self.N, pin)
        self.reset_order()
        self.push()

    # -- weave-time addresses (arena mode) ----------------------------------
    def bake_env(self, weaver: str, base_env: dict | None = None) -> dict:
        if self.arena is None:
            raise RuntimeError("bake_env needs the arena mode (fixed addresses)")
        return compute_bake_env(self.arena.base, self.N, weaver, base_env or os.environ,
                                timer_indirect=self._timer_dev is not None,
                                order_indirect=self._order_dev is not None)

    def arm_process_env(self, weaver: str) -> None:
        env = self.bake_env(weaver)
        for k in self.BAKE_KEYS:
            if k in env:
                os.environ[k] = env[k]
            else:
                os.environ.pop(k, None)

    def use_device_timer(self) -> None:
        """Arena mode: the TIMER word becomes a pointer to a device row table
        (device atomics instead of PCIe atomics). Word 0 means timer off."""
        if self.arena is None:
            return  # device mode already keeps the timer in device memory
        if self._timer_dev is None:
            self._timer_dev = torch.zeros(self.N, dtype=torch.int64, device=self.dev)
            self._timer_stream = torch.cuda.Stream() if self.dev.startswith("cuda") else None
        self.arena.write(TIMER_OFF, struct.pack("<Q", self._timer_dev.data_ptr()))

    def use_device_order(self) -> None:
        """Arena mode: the ORDER word becomes a pointer to a device order
        tensor, so orders install device-to-device without a host sync."""
        if self.arena is None:
            return
        if self._order_dev is None:
            self._order_dev = torch.arange(self.N, dtype=torch.int32, device=self.dev)
        self.arena.write(ORDER_OFF, struct.pack("<Q", self._order_dev.data_ptr()))

    # -- pi --------------------------------------------------------------------
    def set_order(self, tasks) -> None:
        """tasks[i] = the task served by the i-th raw slot (a prefix; the rest
        of the table keeps its previous content, identity after reset)."""
        if isinstance(tasks, torch.Tensor) and tasks.is_cuda and self.mode == "device":
            n = min(tasks.numel(), self.N)
            self.order_t[:n].copy_(tasks[:n].to(torch.int32), non_blocking=True)
            return
        t = torch.as_tensor(tasks, dtype=torch.int32)
        n = min(t.numel(), self.N)
        if self.mode == "device":
            buf = self._order_ring.stage(t[:n].cpu().numpy().tobytes())
            self.order_t[:n].copy_(buf.view(torch.int32)[:n], non_blocking=True)
            self._order_ring.mark()
        elif self._order_dev is not None:
            self._order_dev[:n] = t[:n].to(self._order_dev.device, non_blocking=True)
        else:
            self.arena.write(ORDER_OFF, t[:n].cpu().numpy().tobytes())

    def reset_order(self) -> None:
        self.set_order(torch.arange(self.N, dtype=torch.int32))

    def set_order_size(self, n: int) -> None:
        struct.pack_into("<I", self._ctrl_host, CTRL_ORDER_SIZE_OFF, int(n))

    def install_order(self, tasks, n: int, validate: bool = True) -> None:
        """Concurrent-safe install: the table first, the validity stamp
        (order_size) with the next push. A batch larger than the table raises
        (never truncated), and a host-side order that is not a permutation of
        [0, n) raises before anything is written (a duplicate entry would run
        one task twice and drop another). Device tensors are not inspected:
        that would synchronise the stream."""
        n = int(n)
        if n > self.N:
            raise RuntimeError(f"batch of {n} tasks exceeds the control tables' capacity "
                               f"(SCHED_MAX_TASKS={self.N}); raise max_tasks")
        if validate and not (isinstance(tasks, torch.Tensor) and tasks.is_cuda):
            import numpy as np
            t = np.asarray(torch.as_tensor(tasks).cpu(), dtype=np.int64)[:n]
            if t.size != n or (n and (t.min() < 0 or t.max() >= n or
                                      np.bincount(t, minlength=n).max() != 1)):
                raise ValueError(f"order is not a permutation of [0, {n}): refusing to install it")
        self.set_order(tasks)
        self.set_order_size(n)

    # -- control block ---------------------------------------------------------
    def set_lambda(self, bw=0.0, l2=0.0, smem=0.0, comp=0.0) -> None:
        struct.pack_into("<4f", self._ctrl_host, CTRL_LAMBDA_OFF, float(bw), float(l2),
                         float(smem), float(comp))

    def set_num_tasks(self, n: int) -> None:
        """Work-queue arming switch: 0 = static path, n > 0 = claim loop over n tasks."""
        struct.pack_into("<I", self._ctrl_host, CTRL_NUM_TASKS_OFF, int(n))

    def set_timer_enabled(self, on: bool) -> None:
        (flags,) = struct.unpack_from("<I", self._ctrl_host, CTRL_FLAGS_OFF)
        flags = (flags & ~FLAG_TIMER_OFF) | (0 if on else FLAG_TIMER_OFF)
        struct.pack_into("<I", self._ctrl_host, CTRL_FLAGS_OFF, flags)

    def set_row(self, i: int, q: float = 0.0, tau: int = 0, hint: int = HINT_AUTO) -> None:
        if not 0 <= i < self.N:
            raise IndexError(f"row {i} outside the table ({self.N})")
        struct.pack_into("<fHB", self._ctrl_host, CTRL_ROWS_OFF + ROW_SIZE * i, float(q),
                         int(tau) & 0xFFFF, int(hint) & 0xFF)

    def set_rows(self, q=None, tau=None, hint=None, n: int | None = None) -> None:
        """Vectorised row write: q (f32), tau (u16), hint (u8) for rows [0, n)."""
        n = self.N if n is None else min(int(n), self.N)
        import numpy as np
        rows = np.zeros(n, dtype=np.dtype([("q", "<f4"), ("tau", "<u2"), ("hint", "u1"), ("pad", "u1")]))
        if q is not None:
            rows["q"] = np.asarray(torch.as_tensor(q, dtype=torch.float32).cpu())[:n]
        if tau is not None:
            rows["tau"] = np.clip(np.asarray(torch.as_tensor(tau).cpu(), dtype=np.int64)[:n], 0, 0xFFFF)
        if hint is not None:
            rows["hint"] = np.asarray(torch.as_tensor(hint).cpu(), dtype=np.int64)[:n] & 0xFF
        self._ctrl_host[CTRL_ROWS_OFF:CTRL_ROWS_OFF + ROW_SIZE * n] = rows.tobytes()

    def push(self) -> None:
        """Publish the control mirror with a new generation. Body first, the
        generation word last, so a reader that sees the new generation sees
        complete rows (x86 store order / stream order)."""
        self._generation = (self._generation + 1) & 0xFFFFFFFF
        struct.pack_into("<I", self._ctrl_host, 0, self._generation)
        if self.mode == "device":
            buf = self._ctrl_ring.stage(self._ctrl_host)
            self.ctrl_t[4:].copy_(buf[4:], non_blocking=True)
            self.ctrl_t[:4].copy_(buf[:4], non_blocking=True)
            self._ctrl_ring.mark()
        else:
            self.arena.write(CTRL_OFF + 4, bytes(self._ctrl_host[4:]))
            self.arena.write(CTRL_OFF, bytes(self._ctrl_host[:4]))

    @property
    def generation(self) -> int:
        return self._generation

    def ctrl_snapshot(self) -> bytes:
        return bytes(self._ctrl_host)

    # -- timer -------------------------------------------------------------------
    def clear_timer(self) -> None:
        if self.mode == "device":
            self.timer_t.zero_()
        elif self._timer_dev is not None:
            self._timer_dev.zero_()
        else:
            self.arena.memset(TIMER_OFF, 0, 8 * self.N)

    def read_timer(self) -> torch.Tensor:
        """Per-task cycles. The caller guarantees the writing kernels finished."""
        if self.mode == "device":
            return self.timer_t.to("cpu")
        if self._timer_dev is not None:
            if self._timer_stream is not None:
                with torch.cuda.stream(self._timer_stream):
                    t = self._timer_dev.to("cpu", non_blocking=True)
                self._timer_stream.synchronize()
                return t
            return self._timer_dev.cpu()
        return torch.frombuffer(bytearray(self.arena.read(TIMER_OFF, 8 * self.N)), dtype=torch.int64)

    # -- ticket queue ---------------------------------------------------------------
    def reset_queue(self, workers: int = 0) -> None:
        """Arena mode: prime the ticket for an IR-woven launch of ``workers``
        CTAs (reference semantics). Device mode: the framework's kernels reset
        their own queue on exit; this only zeroes it."""
        if self.mode == "device":
            self.queue_t.zero_()
        else:
            self.arena.write(QUEUE_OFF, struct.pack("<i", int(workers)))

    # -- slots for this framework's kernels -------------------------------------------
    def slots(self) -> dict:
        """Keyword arguments (order, ctrl, timer, queue, max_tasks) for the
        kernel ops. In arena mode the pointers are the host-mapped windows."""
        if self.mode == "device":
            return dict(order=self.order_t, ctrl=self.ctrl_t, timer=self.timer_t,
                        queue=self.queue_t, max_tasks=self.N)
        raise RuntimeError("arena-mode tables are consumed by IR-woven kernels via baked "
                           "addresses; use mode='device' for the framework's kernels")

    # -- R: the resident prefix of a launch ------------------------------------------------
    def sm_count(self) -> int:
        if not self.dev.startswith("cuda"):
            return 0
        return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count

    def r_from_occupancy(self, blocks_per_sm: int) -> int:
        return int(blocks_per_sm) * self.sm_count()

    def r_for_kernel(self, group: int = 4) -> int:
        """R of this framework's woven decode kernel: its occupancy (runtime
        occupancy query on our own kernel) times the SM count."""
        from .._ext import ext
        return self.r_from_occupancy(ext().attn_decode_occupancy(group))

    # -- orders -----------------------------------------------------------------------
    @staticmethod
    def _grouped_lpt(c, block: int) -> torch.Tensor:
        """LPT over blocks of ``block`` adjacent tasks: blocks by descending
        total cost, ascending index inside a block (block=1: plain LPT).
        Coarse blocks keep neighbouring tasks (neighbouring KV) together."""
        c = torch.as_tensor(c).float()
        n = c.numel()
        if block <= 1 or n <= block:
            return torch.argsort(c, descending=True, stable=True).to(torch.int32)
        nb = (n + block - 1) // block
        pad = nb * block - n
        cc = torch.cat([c, c.new_zeros(pad)]) if pad else c
        border = torch.argsort(cc.reshape(nb, block).sum(1), descending=True, stable=True)
        idx = (border[:, None] * block + torch.arange(block)[None, :]).flatten()
        return idx[idx < n].to(torch.int32)

    @staticmethod
    def region_order(cost, R: int, block: int | None = None) -> torch.Tensor:
        """Order for a launch whose first R raw slots start at once and whose
        remaining slots are handed out as workers free up (cluster launch
        control). Prefix: heaviest and lightest tasks alternate, so heavy work
        starts early and light work frees workers quickly; suffix: the rest,
        heaviest first. Without such a split (R <= 0 or n <= R) it is grouped
        LPT with ``block`` (SCHED_LPT_BLOCK, default 16)."""
        c = torch.as_tensor(cost).float()
        n = c.numel()
        if R <= 0 or n <= int(R):
            if block is None:
                block = int(os.environ.get("SCHED_LPT_BLOCK", "16"))
            return SchedPlane._grouped_lpt(c, block)
        R = int(R)
        lpt = torch.argsort(c, descending=True, stable=True).to(torch.int32)
        nh = (R + 1) // 2
        nl = R - nh
        pre = torch.empty(R, dtype=torch.int32)
        pre[0::2] = lpt[:nh]
        if nl:
            pre[1::2] = lpt[n - nl:].flip(0)
        suf = lpt[nh:n - nl] if nl else lpt[nh:]
        return torch.cat([pre, suf])
