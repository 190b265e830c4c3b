// sched/weave.cuh -- source-level weave points for hand-written sm_100a kernels.
//
// nvcc has no pass-plugin interface, so kernels in this framework carry the
// levers as explicit, declared weave points instead of having an IR pass
// insert them. Each function below is the device-side semantics of one
// manifest row (sched/manifest.h), with the same fail-safe rules as the IR
// weaver (csrc/weave): a null slot means "stock behaviour" and every table
// read is bounds-checked, so a disarmed kernel computes exactly what the
// unwoven kernel computes.
//
// Semantics follow the reference pass (lib/SchedWeave.cpp:444-526 remap,
// :532-581 policy flags, :585-614 budget, :979-1049 timer; the work-queue
// driver of lib/SchedWorkQueue.cpp:345-448), re-expressed for kernels that
// receive SchedSlots by value.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "sched/abi.h"

namespace sched {

// Compile-time lever set of one kernel instantiation. Compiled-out levers
// cost nothing; compiled-in levers are still gated by their runtime slots.
struct LeverSet {
  bool pi, shed, policy, timer, pdl;
};
constexpr LeverSet kAllLevers{true, true, true, true, false};
constexpr LeverSet kNoLevers{false, false, false, false, false};

enum class Acquire : int { Static = 0, Ticket = 1, Clc = 2 };

// Marginal-exchange constants of the policy score (reference defaults).
struct PolicyConsts {
  float dT = 1.0f, dR = 1.0f, H = 0.25f;
};

__device__ __forceinline__ const SchedPolicyRow *row_ptr(const SchedCtrl *c, uint32_t i) {
  return reinterpret_cast<const SchedPolicyRow *>(reinterpret_cast<const char *>(c) +
                                                  SCHED_CTRL_ROWS_OFF) + i;
}

// pi: the task served by raw slot `raw` of a launch of `n_launch` tasks.
// Falls back to raw when unarmed, when raw is outside the table, when the
// mapped entry is outside the launch, or -- for the whole launch -- when the
// installed order was built for a different task count.
__device__ __forceinline__ uint32_t remap(const SchedSlots &s, uint32_t raw, uint32_t n_launch) {
  if (s.order == nullptr || raw >= s.max_tasks) return raw;
  uint32_t mapped = (uint32_t)__ldg(s.order + raw);
  bool size_ok = true;
  if (s.ctrl != nullptr) {
    uint32_t osz = __ldg(&s.ctrl->order_size);
    size_ok = (osz == 0u) || (osz == n_launch);
  }
  return (mapped < n_launch && size_ok) ? mapped : raw;
}

// shed: KV units the task may attend; 0xFFFFFFFF = unbounded.
__device__ __forceinline__ uint32_t budget(const SchedSlots &s, uint32_t task) {
  if (s.ctrl == nullptr || task >= s.max_tasks) return 0xFFFFFFFFu;
  uint32_t tau = __ldg(&row_ptr(s.ctrl, task)->tau);
  return tau == 0u ? 0xFFFFFFFFu : tau;
}

struct PolicyFlags {
  bool urgent, polite;
};

// policy: urgent = hint URGENT, or hint AUTO with q*dT - lambda_bw*dR - H > 0;
// polite = hint POLITE. Unarmed / out of range: neither.
__device__ __forceinline__ PolicyFlags policy(const SchedSlots &s, uint32_t task,
                                              PolicyConsts pc = PolicyConsts()) {
  PolicyFlags f{false, false};
  if (s.ctrl == nullptr || task >= s.max_tasks) return f;
  const SchedPolicyRow *r = row_ptr(s.ctrl, task);
  float q = __ldg(&r->q);
  uint8_t hint = __ldg(&r->hint);
  float lam = __ldg(&s.ctrl->lambda[0]);
  float score = q * pc.dT - lam * pc.dR - pc.H;
  f.urgent = hint == SCHED_HINT_URGENT || (hint == SCHED_HINT_AUTO && score > 0.0f);
  f.polite = hint == SCHED_HINT_POLITE;
  return f;
}

// timer: read the off-flag once, at entry; it decides this launch's write.
__device__ __forceinline__ bool timer_off_at_entry(const SchedSlots &s) {
  if (s.timer == nullptr) return true;
  if (s.ctrl == nullptr) return false;
  return (__ldg(&s.ctrl->flags) & SCHED_CTRL_FLAG_TIMER_OFF) != 0u;
}

__device__ __forceinline__ unsigned long long clock_now() {
  unsigned long long c;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
  return c;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Called by one thread per task: commutative add of the task's cycles.
__device__ __forceinline__ void timer_commit(const SchedSlots &s, bool off, uint32_t task,
                                             unsigned long long t0) {
  if (off || s.timer == nullptr || task >= s.max_tasks) return;
  atomicAdd(s.timer + task, clock_now() - t0);
}

// L2 hints for a stream of bytes the task is about to read / has consumed.
__device__ __forceinline__ void l2_prefetch_evict_last(const void *p) {
  asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p));
}
// Polite tier: demote a consumed 128-byte line to normal eviction priority.
// (discard.global.L2 is not used: it drops the line without write-back, so
// data still dirty in L2 would be lost.)
__device__ __forceinline__ void l2_demote_line(const void *p) {
  const void *a = reinterpret_cast<const void *>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(127));
  asm volatile("applypriority.global.L2::evict_normal [%0], 128;" ::"l"(a) : "memory");
}

// PDL overlap points.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;");
}

// Number of tasks of the claim loop this step; 0 means "static path".
__device__ __forceinline__ uint32_t wq_num_tasks(const SchedSlots &s) {
  return s.ctrl == nullptr ? 0u : __ldg(&s.ctrl->num_tasks);
}

// Ticket claim by one thread: next raw task id.
__device__ __forceinline__ uint32_t claim_ticket(const SchedSlots &s) {
  return atomicAdd(s.queue, 1u);
}

// Cluster-launch-control claim by one thread of the CTA. Steals a CTA of this
// grid that has not been launched yet and returns its blockIdx.x, or
// `fallback` when none is left. `result` is a 16-byte aligned shared buffer,
// `mbar` a shared mbarrier initialised once by the caller with count 1;
// `phase` is the caller's parity bit for that mbarrier (flipped on every use).
// The wait is bounded by `budget_ns` of wall time: when it runs out the claim
// reports `fallback` and sets *timed_out, so a lost response ends the loop
// instead of hanging the kernel. After a failed claim (no CTA left) the
// caller must not claim again.
__device__ __forceinline__ uint32_t claim_clc(uint4 *result, uint64_t *mbar, uint32_t &phase,
                                              uint32_t fallback, unsigned long long budget_ns,
                                              bool *timed_out) {
  uint32_t res = static_cast<uint32_t>(__cvta_generic_to_shared(result));
  uint32_t bar = static_cast<uint32_t>(__cvta_generic_to_shared(mbar));
  asm volatile(
      "{\n"
      ".reg .b64 st;\n"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%1], 16;\n"
      "clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], "
      "[%1];\n"
      "}\n" ::"r"(res),
      "r"(bar)
      : "memory");
  const unsigned long long t0 = globaltimer_ns();
  uint32_t done = 0;
  for (uint32_t polls = 0; !done; ++polls) {
    asm volatile(
        "{\n.reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(phase)
        : "memory");
    if (!done && (polls & 255u) == 255u && globaltimer_ns() - t0 > budget_ns) {
      *timed_out = true;
      return fallback;
    }
  }
  phase ^= 1u;
  uint32_t x = fallback, ok = 0;
  asm volatile(
      "{\n.reg .pred p;\n.reg .b128 h;\n"
      "ld.shared.b128 h, [%2];\n"
      "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, h;\n"
      "selp.u32 %1, 1, 0, p;\n"
      "@p clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %0, h;\n"
      "}\n"
      : "+r"(x), "=r"(ok)
      : "r"(res)
      : "memory");
  return ok ? x : fallback;
}

}  // namespace sched
