// sched/sched_rt.h -- host-application runtime contract (named-global ABI).
//
// Applications whose kernels were woven by `sched-weave` (the IR weaver) find
// the control tables through four device globals with fixed names. This
// header defines them and the host API that arms, programs and disarms them.
// The names, the arm/disarm/setter functions and the JSON publication file
// keep the contract of the reference's runtime/sched_rt.h:89-275, so host
// apps written for it link against this one unchanged.
//
// Include it in exactly one CUDA translation unit of the application (it
// defines the device globals). Kernels that are not IR-woven -- every kernel
// in this framework -- take the same tables by value as a SchedSlots launch
// parameter; sched_rt_slots() returns them.
//
// Design differences from the reference, all ABI-neutral:
//   * the timer lives in device memory by default (device atomics cost
//     nothing measurable; host-mapped PCIe atomics cost ~25% on the
//     reference's hardware); sched_rt_init_mapped_timer() keeps the
//     host-mapped zero-touch variant for external observers;
//   * sched_rt_push_ctrl_async() publishes on a stream (graph-capturable)
//     from a pinned host mirror, so a serving loop never synchronises.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <unistd.h>

#include "sched/abi.h"

extern "C" {
__device__ int32_t *__sched_task_order = nullptr;
__device__ SchedCtrl *__sched_ctrl = nullptr;
__device__ unsigned long long *__sched_timer = nullptr;
__device__ uint32_t *__sched_queue = nullptr;
}

namespace sched_rt_detail {

struct State {
  int32_t *order = nullptr;            // device
  SchedCtrl *ctrl = nullptr;           // device
  SchedCtrl *mirror = nullptr;         // pinned host mirror
  unsigned long long *timer = nullptr; // device (or device view of mapped)
  unsigned long long *timer_host = nullptr;  // host view when mapped
  uint32_t *queue = nullptr;           // device
  bool mapped_timer = false;
  bool armed = false;
};

inline State &state() {
  static State s;
  return s;
}

inline bool check(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return true;
  std::fprintf(stderr, "[sched_rt] %s: %s\n", what, cudaGetErrorString(e));
  return false;
}

inline bool publish_slots(int32_t *o, SchedCtrl *c, unsigned long long *t, uint32_t *q) {
  return check(cudaMemcpyToSymbol(__sched_task_order, &o, sizeof(o)), "arm order") &&
         check(cudaMemcpyToSymbol(__sched_ctrl, &c, sizeof(c)), "arm ctrl") &&
         check(cudaMemcpyToSymbol(__sched_timer, &t, sizeof(t)), "arm timer") &&
         check(cudaMemcpyToSymbol(__sched_queue, &q, sizeof(q)), "arm queue");
}

inline void write_json() {
  State &s = state();
  char path[128];
  std::snprintf(path, sizeof(path), "/tmp/sched_rt_%d.json", (int)getpid());
  FILE *f = std::fopen(path, "w");
  if (!f) return;
  std::fprintf(f,
               "{\"pid\":%d,\"max_tasks\":%d,\"order_dev\":%llu,\"ctrl_dev\":%llu,"
               "\"timer_host_va\":%llu,\"timer_bytes\":%zu,\"queue_dev\":%llu}\n",
               (int)getpid(), SCHED_MAX_TASKS, (unsigned long long)(uintptr_t)s.order,
               (unsigned long long)(uintptr_t)s.ctrl,
               (unsigned long long)(uintptr_t)(s.mapped_timer ? (void *)s.timer_host
                                                               : (void *)s.timer),
               (size_t)SCHED_MAX_TASKS * sizeof(unsigned long long),
               (unsigned long long)(uintptr_t)s.queue);
  std::fclose(f);
}

inline bool allocate(bool mapped_timer) {
  State &s = state();
  const size_t n = SCHED_MAX_TASKS;
  if (!check(cudaMalloc(&s.order, n * sizeof(int32_t)), "alloc order")) return false;
  int32_t *ident = static_cast<int32_t *>(std::malloc(n * sizeof(int32_t)));
  for (size_t i = 0; i < n; ++i) ident[i] = (int32_t)i;
  bool ok = check(cudaMemcpy(s.order, ident, n * sizeof(int32_t), cudaMemcpyHostToDevice),
                  "identity order");
  std::free(ident);
  if (!ok) return false;
  if (!check(cudaMallocHost(&s.mirror, sizeof(SchedCtrl)), "alloc mirror")) return false;
  std::memset(s.mirror, 0, sizeof(SchedCtrl));
  if (!check(cudaMalloc(&s.ctrl, sizeof(SchedCtrl)), "alloc ctrl")) return false;
  if (!check(cudaMemcpy(s.ctrl, s.mirror, sizeof(SchedCtrl), cudaMemcpyHostToDevice), "ctrl"))
    return false;
  s.mapped_timer = mapped_timer;
  if (mapped_timer) {
    if (!check(cudaHostAlloc(&s.timer_host, n * 8, cudaHostAllocMapped), "alloc timer"))
      return false;
    std::memset(s.timer_host, 0, n * 8);
    if (!check(cudaHostGetDevicePointer(&s.timer, s.timer_host, 0), "timer devptr"))
      return false;
  } else {
    if (!check(cudaMalloc(&s.timer, n * 8), "alloc timer")) return false;
    if (!check(cudaMemset(s.timer, 0, n * 8), "zero timer")) return false;
  }
  if (!check(cudaMalloc(&s.queue, sizeof(uint32_t)), "alloc queue")) return false;
  return check(cudaMemset(s.queue, 0, sizeof(uint32_t)), "zero queue");
}

inline bool init(bool mapped_timer) {
  State &s = state();
  if (s.armed) return true;
  // Re-arm after a disarm reuses the live buffers: disarm only nulls slots.
  if (!s.order && !allocate(mapped_timer)) return false;
  if (!publish_slots(s.order, s.ctrl, s.timer, s.queue)) return false;
  write_json();
  s.armed = true;
  return true;
}

}  // namespace sched_rt_detail

// Allocate the tables (identity order, neutral ctrl, zero timer), arm the
// device slots and publish /tmp/sched_rt_<pid>.json.
static inline bool sched_rt_init() { return sched_rt_detail::init(false); }
// Same, with the timer in host-mapped pinned memory (read with no CUDA call).
static inline bool sched_rt_init_mapped_timer() { return sched_rt_detail::init(true); }

// Null every slot: woven kernels take their stock path. Reversible.
static inline bool sched_rt_disarm() {
  if (!sched_rt_detail::publish_slots(nullptr, nullptr, nullptr, nullptr)) return false;
  sched_rt_detail::state().armed = false;
  return true;
}

static inline bool sched_rt_set_order(const int32_t *order, unsigned n) {
  if (n > SCHED_MAX_TASKS) n = SCHED_MAX_TASKS;
  return sched_rt_detail::check(cudaMemcpy(sched_rt_detail::state().order, order,
                                           n * sizeof(int32_t), cudaMemcpyHostToDevice),
                                "set order");
}
static inline void sched_rt_set_lambda(float bw, float l2, float smem, float comp) {
  float *l = sched_rt_detail::state().mirror->lambda;
  l[0] = bw, l[1] = l2, l[2] = smem, l[3] = comp;
}
static inline void sched_rt_set_task(unsigned i, float q, uint16_t tau, uint8_t hint) {
  if (i < SCHED_MAX_TASKS) sched_rt_detail::state().mirror->task[i] = {q, tau, hint, 0};
}
static inline void sched_rt_set_tau(unsigned i, uint16_t tau) {
  if (i < SCHED_MAX_TASKS) sched_rt_detail::state().mirror->task[i].tau = tau;
}
static inline void sched_rt_set_num_tasks(uint32_t n) {
  sched_rt_detail::state().mirror->num_tasks = n;
}
static inline void sched_rt_set_order_size(uint32_t n) {
  sched_rt_detail::state().mirror->order_size = n;
}
static inline void sched_rt_set_timer_enabled(bool on) {
  uint32_t &f = sched_rt_detail::state().mirror->flags;
  f = on ? (f & ~SCHED_CTRL_FLAG_TIMER_OFF) : (f | SCHED_CTRL_FLAG_TIMER_OFF);
}

// Publish the mirror (generation bumped). Synchronous form: whole struct.
static inline bool sched_rt_push_ctrl() {
  auto &s = sched_rt_detail::state();
  s.mirror->generation++;
  return sched_rt_detail::check(
      cudaMemcpy(s.ctrl, s.mirror, sizeof(SchedCtrl), cudaMemcpyHostToDevice), "push ctrl");
}
// Stream-ordered form: body first, generation word last, both async.
static inline bool sched_rt_push_ctrl_async(cudaStream_t st) {
  auto &s = sched_rt_detail::state();
  s.mirror->generation++;
  const char *src = reinterpret_cast<const char *>(s.mirror);
  char *dst = reinterpret_cast<char *>(s.ctrl);
  return sched_rt_detail::check(cudaMemcpyAsync(dst + 4, src + 4, sizeof(SchedCtrl) - 4,
                                                cudaMemcpyHostToDevice, st),
                                "push body") &&
         sched_rt_detail::check(cudaMemcpyAsync(dst, src, 4, cudaMemcpyHostToDevice, st),
                                "push generation");
}

// Prime the ticket counter for a launch of `workers` persistent CTAs.
static inline bool sched_rt_queue_reset(uint32_t workers) {
  return sched_rt_detail::check(cudaMemcpy(sched_rt_detail::state().queue, &workers,
                                           sizeof(workers), cudaMemcpyHostToDevice),
                                "queue reset");
}

static inline unsigned long long sched_rt_timer(unsigned i) {
  auto &s = sched_rt_detail::state();
  if (i >= SCHED_MAX_TASKS || !s.timer) return 0ull;
  if (s.mapped_timer) return s.timer_host[i];
  unsigned long long v = 0;
  cudaMemcpy(&v, s.timer + i, 8, cudaMemcpyDeviceToHost);
  return v;
}
static inline void sched_rt_timer_clear() {
  auto &s = sched_rt_detail::state();
  if (!s.timer) return;
  if (s.mapped_timer)
    std::memset(s.timer_host, 0, (size_t)SCHED_MAX_TASKS * 8);
  else
    cudaMemset(s.timer, 0, (size_t)SCHED_MAX_TASKS * 8);
}

// The same tables as a by-value launch parameter for non-woven kernels.
static inline SchedSlots sched_rt_slots() {
  auto &s = sched_rt_detail::state();
  SchedSlots sl{};
  if (s.armed) {
    sl.order = s.order;
    sl.ctrl = s.ctrl;
    sl.timer = s.timer;
    sl.queue = s.queue;
    sl.max_tasks = SCHED_MAX_TASKS;
  }
  return sl;
}
