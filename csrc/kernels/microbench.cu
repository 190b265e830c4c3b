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
// 3. mix_probe: a reused set R read over and over, interleaved 1:1 with a
//    stream S read once (S >> L2). Mode 0 is plain loads (L2's default
//    replacement); mode 1 pins a fraction f of R's lines (evict_last, the
//    rest evict_unchanged) and streams S evict_first; mode 2 is mode 1 with
//    the unpinned part of R evict_first too. Sweeping |R| asks whether cache
//    management pays when a reused set is flooded by a stream (the
//    reference's test/cache_reuse.cu:1-45); sweeping f on an R larger than
//    L2 asks whether residency is a continuous per-request budget (its
//    test/cache_budget.cu:1-32).
// 5. clc_probe: the behaviour of cluster launch control as CTA code sees
//    it, one CTA per task (the grid is the task list). Every CTA runs its
//    task (a %clock64 burn of work[task] cycles), then claims: late bound
//    (try_cancel issued only once the body finished) or claim-ahead (the next
//    try_cancel issued before the body, its answer collected after). Each
//    claim is recorded with the cycles the CTA waited for the answer and the
//    cancelled CTA's id (or a failure), so the host measures the claim
//    latency, checks that every worker ends with exactly one failed claim
//    and that every task ran once, and compares the makespan of the two
//    placements with a static persistent grid (the reference's
//    experiments/clc/FINDINGS.md:203-225 terminal-failure rule, :668-670
//    claim latency, :1244-1256 claim-ahead vs late binding, re-measured on
//    B200).
// 4. pdl_producer / pdl_consumer: two dependent kernels on one stream. The
//    producer releases its dependents at entry; the consumer runs an
//    independent prologue, then griddepcontrol.wait, then reads what the
//    producer wrote. With programmatic stream serialization the prologue and
//    the consumer's launch overlap the producer; results must not change
//    (the reference's test/pdl_overlap.cu:1-70 gates).
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

// ---------------------------------------------------------------- clc
struct ClcArgs {
  const uint32_t *work;       // per task: cycles of the body
  int n_tasks;
  int mode;                   // 0 static persistent grid, 1 CLC late bound, 2 CLC claim-ahead
  int max_rec;                // claim records per CTA
  unsigned *hits;             // [n_tasks] executions (must end at 1)
  unsigned long long *rec;    // [grid][max_rec]: waited cycles << 32 | (cancelled CTA id, or ~0u on failure)
  unsigned *n_rec;            // [grid] claims recorded per CTA
  unsigned *smid;             // [grid] SM of each CTA
  int *status;
};

__device__ __forceinline__ void clc_body(const ClcArgs &a, int task) {
  if (threadIdx.x == 0) {
    const long long t0 = clock64();
    while (clock64() - t0 < (long long)a.work[task]) {
    }
    atomicAdd(a.hits + task, 1u);
  }
  __syncthreads();
}

__device__ __forceinline__ void clc_issue(uint4 *result, uint64_t *bar) {
  const uint32_t res = static_cast<uint32_t>(__cvta_generic_to_shared(result));
  const uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
  asm volatile(
      "{\n.reg .b64 st;\n"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%1], 16;\n"
      "clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], [%1];\n"
      "}\n" ::"r"(res),
      "r"(b)
      : "memory");
}

// Waits (bounded) for the answer of the claim in flight; returns the
// cancelled CTA's x id or ~0u (failure, or the wait gave up).
__device__ __forceinline__ uint32_t clc_collect(uint4 *result, uint64_t *bar, uint32_t &phase, int *status) {
  const uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
  const uint64_t t0 = ptx::globaltimer_ns();
  uint32_t done = 0;
  for (uint32_t polls = 0; !done; ++polls) {
    asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(done)
                 : "r"(b), "r"(phase)
                 : "memory");
    if (!done && (polls & 255u) == 255u && ptx::globaltimer_ns() - t0 > kWaitBudgetNs) {
      report_status(status, kStatusClcTimeout);
      return ~0u;
    }
  }
  phase ^= 1u;
  uint32_t x = ~0u;
  const uint32_t res = static_cast<uint32_t>(__cvta_generic_to_shared(result));
  asm volatile(
      "{\n.reg .pred p;\n.reg .b128 h;\n"
      "ld.shared.b128 h, [%1];\n"
      "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, h;\n"
      "@p clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %0, h;\n"
      "}\n"
      : "+r"(x)
      : "r"(res)
      : "memory");
  return x;
}

__global__ void __launch_bounds__(128) clc_probe(const ClcArgs a) {
  __shared__ uint4 result;
  __shared__ uint64_t bar;
  __shared__ uint32_t next;
  const int c = blockIdx.x;
  if (threadIdx.x == 0) a.smid[c] = ptx::smid();
  if (a.mode == 0) {
    for (int t = c; t < a.n_tasks; t += gridDim.x) clc_body(a, t);
    return;
  }
  if (threadIdx.x == 0) {
    ptx::mbar_init(&bar, 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();
  uint32_t phase = 0, nrec = 0;
  uint32_t t = c;
  while (t < (uint32_t)a.n_tasks) {
    if (a.mode == 2 && threadIdx.x == 0) clc_issue(&result, &bar);  // reserve the next task now
    clc_body(a, (int)t);
    if (threadIdx.x == 0) {
      if (a.mode == 1) clc_issue(&result, &bar);  // late binding: claim only when free
      const long long w0 = clock64();
      const uint32_t x = clc_collect(&result, &bar, phase, a.status);
      const unsigned long long waited = (unsigned long long)(clock64() - w0);
      if (nrec < (uint32_t)a.max_rec) a.rec[(size_t)c * a.max_rec + nrec] = (waited << 32) | x;
      ++nrec;
      next = x;
    }
    __syncthreads();
    t = next;
    __syncthreads();
  }
  if (threadIdx.x == 0) a.n_rec[c] = nrec;
}

// ---------------------------------------------------------------- clc shapes
// The CLC contract under other launch shapes (after the reference's
// experiments/clc/clc_2d_probe.cu, clc_tuple_probe.cu,
// clc_participation_probe.cu, clc_cluster_probe.cu; FINDINGS.md:513-802):
// 2-D / 3-D grids (a claim returns the cancelled CTA's (x, y, z); its linear
// id is x + y gx + z gx gy), partial participation (only CTAs whose linear
// id is a multiple of `stride` claim; the others run their own task and
// leave), and clustered launches (cluster of `cx` CTAs along x: the cluster's
// rank 0 claims once per round for the whole cluster and passes the answer to
// its peers through distributed shared memory; a claim cancels a whole
// cluster, whose CTA k then runs task base + k).
struct ClcShapeArgs {
  const uint32_t *work;  // [n] cycles of each task's body
  int n;                 // tasks = CTAs of the launch
  int gx, gy;            // grid x and y (linear id = x + y gx + z gx gy)
  int stride;            // claim participation: linear id (cluster base) % stride == 0
  int cx;                // cluster size along x (1: no cluster)
  unsigned *hits;        // [n] executions (must end at 1)
  unsigned *claimed;     // [n] times a task came back from a claim
  unsigned *launched;    // [n] 1 when the task's CTA was started by the launcher
  unsigned *fails;       // [n] failed claims of the worker that started as that CTA
  unsigned *w_nonzero;   // fourth word of a claim answer seen non-zero
  int *status;
};

__device__ __forceinline__ void clc_shape_body(const ClcShapeArgs &a, uint32_t task) {
  if (threadIdx.x == 0) {
    const long long t0 = clock64();
    while (clock64() - t0 < (long long)a.work[task]) {
    }
    atomicAdd(a.hits + task, 1u);
  }
  __syncthreads();
}

// Waits (bounded) for the claim in flight; returns the cancelled CTA's
// linear id, or ~0u on failure / give-up.
__device__ __forceinline__ uint32_t clc_collect_linear(uint4 *result, uint64_t *bar, uint32_t &phase,
                                                       const ClcShapeArgs &a) {
  const uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
  const uint64_t t0 = ptx::globaltimer_ns();
  uint32_t done = 0;
  for (uint32_t polls = 0; !done; ++polls) {
    asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(done)
                 : "r"(b), "r"(phase)
                 : "memory");
    if (!done && (polls & 255u) == 255u && ptx::globaltimer_ns() - t0 > kWaitBudgetNs) {
      report_status(a.status, kStatusClcTimeout);
      return ~0u;
    }
  }
  phase ^= 1u;
  uint32_t ok = 0, x = 0, y = 0, z = 0, w = 0;
  const uint32_t res = static_cast<uint32_t>(__cvta_generic_to_shared(result));
  asm volatile(
      "{\n.reg .pred p;\n.reg .b128 h;\n"
      "ld.shared.b128 h, [%5];\n"
      "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, h;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "@p clusterlaunchcontrol.query_cancel.get_first_ctaid.v4.b32.b128 {%1, %2, %3, %4}, h;\n"
      "}\n"
      : "=r"(ok), "+r"(x), "+r"(y), "+r"(z), "+r"(w)
      : "r"(res)
      : "memory");
  if (!ok) return ~0u;
  if (w != 0u) atomicAdd(a.w_nonzero, 1u);
  return x + y * (uint32_t)a.gx + z * (uint32_t)a.gx * (uint32_t)a.gy;
}

__global__ void __launch_bounds__(128) clc_shape_probe(const ClcShapeArgs a) {
  __shared__ uint4 result;
  __shared__ uint64_t bar;
  __shared__ uint32_t next;
  const uint32_t me = blockIdx.x + blockIdx.y * (uint32_t)a.gx + blockIdx.z * (uint32_t)a.gx * (uint32_t)a.gy;
  const uint32_t rank = a.cx > 1 ? ptx::cluster_ctarank() : 0u;
  const uint32_t base = me - rank;  // the cluster's first CTA (clusters run along x)
  if (threadIdx.x == 0) {
    a.launched[me] = 1u;
    ptx::mbar_init(&bar, 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();
  if (a.cx > 1) ptx::cluster_sync_all();  // peers' shared memory is live before any DSMEM store
  clc_shape_body(a, me);
  const bool claims = (base % (uint32_t)a.stride) == 0u;
  if (!claims) return;  // the whole cluster leaves together (same base)
  uint32_t phase = 0, nfail = 0;
  while (true) {
    if (threadIdx.x == 0 && rank == 0u) {
      const uint32_t r = static_cast<uint32_t>(__cvta_generic_to_shared(&result));
      const uint32_t bb = static_cast<uint32_t>(__cvta_generic_to_shared(&bar));
      asm volatile(
          "{\n.reg .b64 st;\n"
          "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%1], 16;\n"
          "clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], [%1];\n"
          "}\n" ::"r"(r),
          "r"(bb)
          : "memory");
      const uint32_t x = clc_collect_linear(&result, &bar, phase, a);
      if (x == ~0u) ++nfail;
      next = x;
      // the cluster's other CTAs read the answer from rank 0's shared memory
      // after the cluster barrier below
    }
    uint32_t t;
    if (a.cx > 1) {
      ptx::cluster_sync_all();  // rank 0's `next` is written
      const uint32_t remote = ptx::mapa_shared(static_cast<uint32_t>(__cvta_generic_to_shared(&next)), 0);
      uint32_t v;
      asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(remote) : "memory");
      t = v;
      ptx::cluster_sync_all();  // everyone has read it before rank 0 overwrites it
    } else {
      __syncthreads();
      t = next;
      __syncthreads();
    }
    if (t == ~0u) break;
    const uint32_t task = t + rank;
    if (threadIdx.x == 0 && task < (uint32_t)a.n) atomicAdd(a.claimed + task, 1u);
    if (task < (uint32_t)a.n) clc_shape_body(a, task);
  }
  if (threadIdx.x == 0 && rank == 0u) a.fails[me] = nfail;
}

// ---------------------------------------------------------------- mix
__device__ __forceinline__ uint4 ld_plain(const uint4 *a) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(a));
  return v;
}

__global__ void __launch_bounds__(512) mix_probe(const uint4 *__restrict__ R, size_t rn,
                                                 const uint4 *__restrict__ S, size_t sn, int mode, float frac,
                                                 unsigned *__restrict__ sink) {
  uint64_t pin = 0, str = 0;
  if (mode == 1)
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, %1;" : "=l"(pin) : "f"(frac));
  else if (mode == 2)
    asm volatile("createpolicy.fractional.L2::evict_last.L2::evict_first.b64 %0, %1;" : "=l"(pin) : "f"(frac));
  if (mode != 0) asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(str));
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t j = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  size_t r = j % rn;
  unsigned acc = 0;
  for (; j < sn; j += stride) {
    uint4 a, b;
    if (mode == 0) {
      a = ld_plain(R + r);
      b = ld_plain(S + j);
    } else {
      a = ld_hint(R + r, pin);
      b = ld_hint(S + j, str);
    }
    acc ^= a.x ^ a.w ^ b.y ^ b.z;
    r += stride;
    while (r >= rn) r -= rn;
  }
  if (acc == 0x9E3779B9u) sink[blockIdx.x] = acc;
}

// ---------------------------------------------------------------- PDL pair
__global__ void __launch_bounds__(256) pdl_producer(float *__restrict__ buf, int n, int work) {
  ptx::pdl_launch_dependents();  // the consumer may launch now; it waits before reading
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float v = (float)(i & 1023) * 1e-3f;
  for (int k = 0; k < work; ++k) v = fmaf(v, 0.999f, 1e-3f);
  buf[i] = v;
}

__global__ void __launch_bounds__(256) pdl_consumer(const float *__restrict__ buf, float *__restrict__ out, int n,
                                                    const float *__restrict__ table, int prologue) {
  // independent prologue: work that does not touch the producer's output
  // (a consumer's control-table reads, its weights)
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  float t = 0.f;
  for (int k = 0; k < prologue; ++k) t = fmaf(t, 0.5f, table[(i + k) & 255]);
  ptx::pdl_wait();
  if (i < n) out[i] = buf[i] * 2.0f + t;
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

extern "C" int sched_probe_clc(const uint32_t *work, int n_tasks, int mode, int grid, int max_rec, unsigned *hits,
                               unsigned long long *rec, unsigned *n_rec, unsigned *smid, int *status,
                               cudaStream_t st) {
  if (n_tasks <= 0 || mode < 0 || mode > 2 || max_rec <= 0) return -1;
  probe::ClcArgs a{};
  a.work = work;
  a.n_tasks = n_tasks;
  a.mode = mode;
  a.max_rec = max_rec;
  a.hits = hits;
  a.rec = rec;
  a.n_rec = n_rec;
  a.smid = smid;
  a.status = status;
  const int g = mode == 0 ? grid : n_tasks;
  if (g <= 0) return -1;
  probe::clc_probe<<<g, 128, 0, st>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

// grid (gx, gy, gz) of 128-thread CTAs, optional cluster of cx CTAs along x
// (gx % cx == 0); every CTA runs its own task first; CTAs whose cluster base
// is a multiple of `stride` then claim until a claim fails.
extern "C" int sched_probe_clc_shape(const uint32_t *work, int gx, int gy, int gz, int stride, int cx,
                                     unsigned *hits, unsigned *claimed, unsigned *launched, unsigned *fails,
                                     unsigned *w_nonzero, int *status, cudaStream_t st) {
  if (gx <= 0 || gy <= 0 || gz <= 0 || stride <= 0 || cx <= 0 || cx > 8 || gx % cx != 0) return -1;
  probe::ClcShapeArgs a{};
  a.work = work;
  a.n = gx * gy * gz;
  a.gx = gx;
  a.gy = gy;
  a.stride = stride;
  a.cx = cx;
  a.hits = hits;
  a.claimed = claimed;
  a.launched = launched;
  a.fails = fails;
  a.w_nonzero = w_nonzero;
  a.status = status;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gx, gy, gz);
  cfg.blockDim = dim3(128);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = cx;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = cx > 1 ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, probe::clc_shape_probe, a) != cudaSuccess) return -4;
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

// Resident clusters of cx CTAs of the shape probe (R_cta = this x cx), or
// resident CTAs (x SMs) when cx = 1.
extern "C" int sched_probe_clc_shape_capacity(int cx) {
  if (cx <= 1) {
    int n = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, probe::clc_shape_probe, 128, 0);
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    return n * sms;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cx * 1024);
  cfg.blockDim = dim3(128);
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = cx;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, probe::clc_shape_probe, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n * cx;
}

// CTAs of the task probe resident per SM (R = this x SMs).
extern "C" int sched_probe_tasks_occupancy() {
  int n = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, probe::task_probe, 128, 0);
  return n;
}

extern "C" int sched_probe_mix(const void *R, size_t r_bytes, const void *S, size_t s_bytes, int mode, float frac,
                               unsigned *sink, int grid, cudaStream_t st) {
  if (r_bytes < 16 || s_bytes < 16 || grid <= 0 || mode < 0 || mode > 2 || !(frac > 0.f && frac <= 1.f)) return -1;
  probe::mix_probe<<<grid, 512, 0, st>>>(static_cast<const uint4 *>(R), r_bytes / 16, static_cast<const uint4 *>(S),
                                         s_bytes / 16, mode, frac, sink);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

// `pairs` producer -> consumer launches back to back on `st`; with pdl the
// consumer is launched with programmatic stream serialization.
extern "C" int sched_probe_pdl_pairs(float *buf, float *out, int n, const float *table, int work, int prologue,
                                     int pdl, int pairs, cudaStream_t st) {
  if (n <= 0 || pairs <= 0) return -1;
  const dim3 grid((n + 255) / 256), block(256);
  for (int it = 0; it < pairs; ++it) {
    probe::pdl_producer<<<grid, block, 0, st>>>(buf, n, work);
    if (pdl) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = grid;
      cfg.blockDim = block;
      cfg.stream = st;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      at[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      if (cudaLaunchKernelEx(&cfg, probe::pdl_consumer, (const float *)buf, out, n, table, prologue) != cudaSuccess)
        return -4;
    } else {
      probe::pdl_consumer<<<grid, block, 0, st>>>(buf, out, n, table, prologue);
    }
  }
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

// One producer launch (for fixtures whose consumer is another module's kernel).
extern "C" int sched_probe_pdl_produce(float *buf, int n, int work, cudaStream_t st) {
  if (n <= 0) return -1;
  probe::pdl_producer<<<(n + 255) / 256, 256, 0, st>>>(buf, n, work);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}
