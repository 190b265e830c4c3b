"""Byte layout of the control tables (mirror of include/sched/abi.h).

Kept bit-compatible with the reference contract (runtime/sched_rt.h:54-86 and
python/sched_rt.py:52-63 of jc-su/sched-pass): a control plane written for it
programs these kernels unchanged.
"""

CTRL_GENERATION_OFF = 0
CTRL_NUM_TASKS_OFF = 4
CTRL_LAMBDA_OFF = 8       # f32[4]: bw, l2, smem, comp
CTRL_FLAGS_OFF = 24       # u32, bit0 = timer off
CTRL_ORDER_SIZE_OFF = 28  # u32, task count the order was built for (0 = unchecked)
CTRL_ROWS_OFF = 32
ROW_SIZE = 8              # f32 q, u16 tau, u8 hint, u8 pad
ROW_Q_OFF = 0
ROW_TAU_OFF = 4
ROW_HINT_OFF = 6
FLAG_TIMER_OFF = 1

HINT_AUTO, HINT_URGENT, HINT_POLITE = 0, 1, 2

# fixed-VA arena (baked ABI)
ORDER_OFF = 0x00000
CTRL_OFF = 0x40000
TIMER_OFF = 0x80000
QUEUE_OFF = 0xC0000
ARENA_BYTES = 0x100000
MAX_TASKS_LIMIT = 16384
DEFAULT_VA_BASE = 0x5C00_0000_0000

DEFAULT_MAX_TASKS = 4096


def ctrl_bytes(max_tasks: int) -> int:
    return CTRL_ROWS_OFF + ROW_SIZE * int(max_tasks)
