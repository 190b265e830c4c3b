// microbench.cu -- hardware probes behind the scheduling levers.
//
// 1. stream_probe: one pass over a buffer larger than L2 with every load
//    under one L2 cache policy (none, evict_first, evict_last, evict_normal,
//    evict_unchanged): the HBM ceiling the policy lever works against, and
//    whether a hint changes it (the reference's test/cache_hint_bw.cu:20-52
//    question, asked of B200's 126 MB L2).
// 2. task_probe: a 1-D grid of tasks whose costs come from an array (a
//    %globaltimer burn of cost[i] ns, or a stream of cost[i] bytes), run
//    three ways -- static grid-stride over R persistent CTAs, a ticket
//    counter over R CTAs, or cluster launch control with one CTA per task
//    (finished CTAs cancel unlaunched ones and run their tasks). Every
//    execution increments hits[task], so the host checks exactly-once
//    coverage; per-CTA task counts and the makespan show the balance (the
//    reference's experiments/clc/clc_probe.cu, clc_membound_probe.cu,
//    clc_noise_probe.cu family, re-measured on B200).
// Every wait here is bounded; nothing spins on another CTA.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "sched/ptx.cuh"
#include "sched/weave.cuh"

namespace probe {

enum Policy : int { kNone = 0, kEvictFirst = 1, kEvictLast = 2, kEvictNormal = 3, kEvictUnchanged = 4 };

__device__ __forceinline__ uint64_t make_policy(int pol) {
  uint64_t p = 0;
  if (pol == kEvictFirst)
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  else if (pol == kEvictLast)
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  else if (pol == kEvictNormal)
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  else if (pol == kEvictUnchanged)
    asm volatile("createpolicy.fractional.L2::evict_unchanged.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint4 ld_hint(const uint4 *a, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(a), "l"(pol));
  return v;
}

__global__ void __launch_bounds__(512) stream_probe(const uint4 *__restrict__ src, size_t n, int pol,
                                                    unsigned *__restrict__ sink) {
  const uint64_t p = make_policy(pol);
  unsigned acc = 0;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  constexpr int U = 4;
  for (; i + (U - 1) * stride < n; i += U * stride) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) v[u] = pol == kNone ? __ldcs(src + i + u * stride) : ld_hint(src + i + u * stride, p);
#pragma unroll
    for (int u = 0; u < U; ++u) acc ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
  }
  for (; i < n; i += stride) {
    const uint4 v = pol == kNone ? __ldcs(src + i) : ld_hint(src + i, p);
    acc ^= v.x ^ v.y ^ v.z ^ v.w;
  }
  if (acc == 0x9E3779B9u) sink[blockIdx.x] = acc;  // keeps the loads alive
}

struct TaskArgs {
  const uint32_t *cost;   // per task: ns of burn, or bytes to stream
  int n_tasks;
  int mode;               // 0 static, 1 ticket, 2 CLC
  int memory;             // 0: time burn, 1: stream cost[i] bytes from `data`
  const uint4 *data;
  size_t data_vec;
  unsigned *hits;         // [n_tasks] executions (must end at 1)
  unsigned *per_cta;      // [grid] tasks run by each CTA
  unsigned *ticket;       // mode 1: claim counter (zero before the launch)
  unsigned *sink;
  int *status;
};

__device__ void run_task(const TaskArgs &a, int task) {
  const uint32_t c = a.cost[task];
  if (!a.memory) {
    if (threadIdx.x == 0) {
      const uint64_t t0 = ptx::globaltimer_ns();
      while (ptx::globaltimer_ns() - t0 < c) {
      }
    }
  } else {
    // stream c bytes starting at a task-dependent offset
    const size_t nvec = c / 16;
    const size_t base = ((size_t)task * 7919u * 64u) % (a.data_vec > nvec ? a.data_vec - nvec : 1);
    unsigned acc = 0;
    for (size_t i = threadIdx.x; i < nvec; i += blockDim.x) {
      const uint4 v = __ldcs(a.data + base + i);
      acc ^= v.x ^ v.w;
    }
    if (acc == 0x9E3779B9u) a.sink[0] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    atomicAdd(a.hits + task, 1u);
    atomicAdd(a.per_cta + blockIdx.x, 1u);
  }
}

__global__ void __launch_bounds__(128) task_probe(const TaskArgs a) {
  __shared__ uint4 clc_result;
  __shared__ uint64_t clc_bar;
  __shared__ int next;
  if (a.mode == 0) {
    for (int t = blockIdx.x; t < a.n_tasks; t += gridDim.x) run_task(a, t);
    return;
  }
  if (a.mode == 1) {
    for (;;) {
      if (threadIdx.x == 0) next = (int)atomicAdd(a.ticket, 1u);
      __syncthreads();
      const int t = next;
      __syncthreads();
      if (t >= a.n_tasks) break;
      run_task(a, t);
    }
    return;
  }
  // mode 2: cluster launch control. Run our own task, then cancel a CTA that
  // has not launched yet and run its task instead; the claim is issued only
  // after the current task finished (late binding).
  if (threadIdx.x == 0) {
    ptx::mbar_init(&clc_bar, 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();
  uint32_t phase = 0;
  int t = blockIdx.x;
  while (t < a.n_tasks) {
    run_task(a, t);
    if (threadIdx.x == 0) {
      bool timed_out = false;
      const uint32_t x = sched::claim_clc(&clc_result, &clc_bar, phase, 0xFFFFFFFFu, kWaitBudgetNs, &timed_out);
      if (timed_out) report_status(a.status, kStatusClcTimeout);
      next = x == 0xFFFFFFFFu ? a.n_tasks : (int)x;
    }
    __syncthreads();
    t = next;
    __syncthreads();
  }
}

}  // namespace probe

extern "C" int sched_probe_stream(const void *src, size_t bytes, int policy, unsigned *sink, int grid,
                                  cudaStream_t st) {
  if (bytes < 16 || grid <= 0) return -1;
  probe::stream_probe<<<grid, 512, 0, st>>>(static_cast<const uint4 *>(src), bytes / 16, policy, sink);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int sched_probe_tasks(const uint32_t *cost, int n_tasks, int mode, int grid, int memory,
                                 const void *data, size_t data_bytes, unsigned *hits, unsigned *per_cta,
                                 unsigned *ticket, unsigned *sink, int *status, cudaStream_t st) {
  if (n_tasks <= 0 || mode < 0 || mode > 2) return -1;
  probe::TaskArgs a{};
  a.cost = cost;
  a.n_tasks = n_tasks;
  a.mode = mode;
  a.memory = memory;
  a.data = static_cast<const uint4 *>(data);
  a.data_vec = data_bytes / 16;
  a.hits = hits;
  a.per_cta = per_cta;
  a.ticket = ticket;
  a.sink = sink;
  a.status = status;
  const int g = mode == 2 ? n_tasks : grid;
  if (g <= 0) return -1;
  probe::task_probe<<<g, 128, 0, st>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

// CTAs of the task probe resident per SM (R = this x SMs).
extern "C" int sched_probe_tasks_occupancy() {
  int n = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, probe::task_probe, 128, 0);
  return n;
}
