// sched/abi.h -- the control-table ABI shared by every side of the framework.
//
// One header, three consumers:
//   * host C++ (the runtime contract in sched_rt.h, the pybind module),
//   * device code (the weave points in weave.cuh read the same structs),
//   * the IR weaver (csrc/weave), which emits raw byte offsets into SchedCtrl.
//
// The layout is bit-compatible with the reference's SchedCtrl /
// SchedPolicyRow (runtime/sched_rt.h:54-86 of jc-su/sched-pass) so that a
// control plane written against that contract drives these kernels unchanged:
//
//   SchedCtrl  @0 generation u32 | @4 num_tasks u32 | @8 lambda f32[4]
//              @24 flags u32 (bit0 = timer off) | @28 order_size u32
//              @32 rows: SchedPolicyRow[max_tasks]
//   SchedPolicyRow (8 B) @0 q f32 | @4 tau u16 | @6 hint u8 | @7 pad
//
// Everything here is plain C (usable from .c, .cpp and .cu translation units).
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifndef SCHED_MAX_TASKS
#define SCHED_MAX_TASKS 4096
#endif

// Arena windows of the fixed-VA (baked) ABI; identical offsets on the Python
// side (sched_pass_b200/runtime/abi.py).
#define SCHED_ARENA_ORDER_OFF 0x00000u
#define SCHED_ARENA_CTRL_OFF 0x40000u
#define SCHED_ARENA_TIMER_OFF 0x80000u
#define SCHED_ARENA_QUEUE_OFF 0xC0000u
#define SCHED_ARENA_BYTES 0x100000u
#define SCHED_ARENA_MAX_TASKS 16384u

#define SCHED_CTRL_GENERATION_OFF 0u
#define SCHED_CTRL_NUM_TASKS_OFF 4u
#define SCHED_CTRL_LAMBDA_OFF 8u
#define SCHED_CTRL_FLAGS_OFF 24u
#define SCHED_CTRL_ORDER_SIZE_OFF 28u
#define SCHED_CTRL_ROWS_OFF 32u
#define SCHED_CTRL_ROW_SIZE 8u
#define SCHED_CTRL_ROW_Q_OFF 0u
#define SCHED_CTRL_ROW_TAU_OFF 4u
#define SCHED_CTRL_ROW_HINT_OFF 6u

#define SCHED_CTRL_FLAG_TIMER_OFF 1u

#define SCHED_HINT_AUTO 0u
#define SCHED_HINT_URGENT 1u
#define SCHED_HINT_POLITE 2u

#ifdef __cplusplus
extern "C" {
#endif

typedef struct SchedPolicyRow {
  float q;       // urgency (>= 0); feeds the prefetch score q*dT - lambda_bw*dR - H
  uint16_t tau;  // shed budget in KV units (tokens for our kernels); 0 = none
  uint8_t hint;  // SCHED_HINT_*: 0 auto (decide by score), 1 urgent, 2 polite
  uint8_t _pad;
} SchedPolicyRow;

// Header of the control block. The rows follow it in memory; the host sizes
// the allocation for its own max_tasks (the arena path allows up to 16384).
typedef struct SchedCtrlHeader {
  uint32_t generation;  // bumped on every publish; written LAST
  uint32_t num_tasks;   // work-queue arming switch: 0 = static (stock) path
  float lambda[4];      // shadow prices {bw, l2, smem, comp}
  uint32_t flags;       // bit0: timer off for this launch
  uint32_t order_size;  // task count the installed order was built for (0 = unchecked)
} SchedCtrlHeader;

// Full control block at the compile-time capacity, for the named-global ABI.
typedef struct SchedCtrl {
  uint32_t generation;
  uint32_t num_tasks;
  float lambda[4];
  uint32_t flags;
  uint32_t order_size;
  SchedPolicyRow task[SCHED_MAX_TASKS];
} SchedCtrl;

// The four runtime slots. Our own kernels take this struct BY VALUE as a
// launch parameter (no device-global indirection, so one process can run
// several independently armed planes and CUDA graphs capture the pointers).
// A null slot disables its lever: null order -> identity, null ctrl -> no
// policy/shed/work-queue, null timer -> no observation.
typedef struct SchedSlots {
  const int32_t *order;             // pi: task = order[raw]
  const SchedCtrl *ctrl;            // header + rows (only max_tasks rows valid)
  unsigned long long *timer;        // per-task cycle accumulator (u64)
  uint32_t *queue;                  // ticket counter for the work queue
  uint32_t max_tasks;               // rows valid in order/ctrl/timer
  uint32_t _pad;
} SchedSlots;

#ifdef __cplusplus
}  // extern "C"

static_assert(offsetof(SchedCtrl, num_tasks) == SCHED_CTRL_NUM_TASKS_OFF, "abi");
static_assert(offsetof(SchedCtrl, lambda) == SCHED_CTRL_LAMBDA_OFF, "abi");
static_assert(offsetof(SchedCtrl, flags) == SCHED_CTRL_FLAGS_OFF, "abi");
static_assert(offsetof(SchedCtrl, order_size) == SCHED_CTRL_ORDER_SIZE_OFF, "abi");
static_assert(offsetof(SchedCtrl, task) == SCHED_CTRL_ROWS_OFF, "abi");
static_assert(sizeof(SchedCtrlHeader) == SCHED_CTRL_ROWS_OFF, "abi");
static_assert(sizeof(SchedPolicyRow) == SCHED_CTRL_ROW_SIZE, "abi");
static_assert(offsetof(SchedPolicyRow, tau) == SCHED_CTRL_ROW_TAU_OFF, "abi");
static_assert(offsetof(SchedPolicyRow, hint) == SCHED_CTRL_ROW_HINT_OFF, "abi");
static_assert(sizeof(SchedSlots) == 40, "abi");
#endif
