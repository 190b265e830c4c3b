// common.cuh -- small shared pieces of the framework's CUDA kernels.
#pragma once

#include <cstdlib>

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

// Status codes written (first writer wins) into a caller-provided device word
// when a bounded wait gives up. 0 = OK. The host reads and clears the word.
enum KernelStatus : int {
  kStatusOk = 0,
  kStatusTmaTimeout = 1,      // a TMA completion never arrived
  kStatusMmaTimeout = 2,      // a tensor-core commit never arrived
  kStatusEpilogueTimeout = 3, // the epilogue never saw its accumulator
  kStatusPeerTimeout = 4,     // a peer GPU's flag never arrived
  kStatusClcTimeout = 5,      // a cluster-launch-control response never arrived
  kStatusBadArgument = 6,
  kStatusBadIndex = 7,        // a caller-provided index was out of range; that access was skipped
};

// Where a bad index came from (status word 1).
enum IndexSite : int {
  kSiteCopySrcPage = 1,   // kv page copy: source page of a pair
  kSiteCopyDstPage = 2,   // kv page copy: destination page of a pair
  kSiteKvSlot = 3,        // KV append: cache slot of a token
  kSiteTokenId = 4,       // embedding: token id
  kSiteDecodePage = 5,    // decode attention: block-table page id
  kSitePrefillPage = 6,   // prefill attention: block-table page id
};

// A status buffer holds 4 int32 words: [0] the code, and for
// kStatusBadIndex [1] the site and [2..3] the offending index (int64) of the
// first fault. Only the thread whose CAS set the code writes words 1-3.
__device__ __forceinline__ void report_status(int *status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

// A timeout with the wait that gave up (word [1]; sites kWait* below).
__device__ __forceinline__ void report_timeout(int *status, int code, int wait_site) {
  if (status == nullptr) return;
  if (atomicCAS(status, 0, code) == 0) status[1] = wait_site;
}
// Decode attention's task-handoff waits (word [1] of a timeout status).
enum WaitSite : int {
  kWaitProducerTaskEmpty = 101,
  kWaitMmaTaskFull = 102,
  kWaitMmaQReady = 103,
  kWaitMmaOFree = 104,
  kWaitSoftmaxTaskFull = 105,
};

__device__ __forceinline__ void report_bad_index(int *status, int site, long long index) {
  if (status == nullptr) return;
  if (atomicCAS(status, 0, kStatusBadIndex) == 0) {
    status[1] = site;
    *reinterpret_cast<long long *>(status + 2) = index;
  }
}

// Wall-time budget (ns) of every bounded wait on an mbarrier or a flag.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

__device__ __forceinline__ float bf16_to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}

// sm_100 scalar-pipe helpers for softmax-style row work: the hardware 2^x
// (MUFU, flush-to-zero; 2^-inf = +0), a three-input max, and packed fp32
// pairs (one instruction for two lanes' worth of FMA / add).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// (x0, x1) = (a0 * b0 + c0, a1 * b1 + c1) for b = (b0, b1) and c = (c0, c1) packed
__device__ __forceinline__ void ffma2(float &x0, float &x1, float a0, float a1, uint64_t b, uint64_t c) {
  asm("{\n.reg .b64 t;\nmov.b64 t, {%2, %3};\nfma.rn.f32x2 t, t, %4, %5;\nmov.b64 {%0, %1}, t;\n}"
      : "=f"(x0), "=f"(x1)
      : "f"(a0), "f"(a1), "l"(b), "l"(c));
}
// (acc0, acc1) += (a0, a1)
__device__ __forceinline__ void fadd2(float &acc0, float &acc1, float a0, float a1) {
  asm("{\n.reg .b64 t, u;\nmov.b64 t, {%0, %1};\nmov.b64 u, {%2, %3};\nadd.rn.f32x2 t, t, u;\n"
      "mov.b64 {%0, %1}, t;\n}"
      : "+f"(acc0), "+f"(acc1)
      : "f"(a0), "f"(a1));
}
__device__ __forceinline__ uint64_t f32x2_splat(float v) {
  const uint32_t u = __float_as_uint(v);
  return ((uint64_t)u << 32) | u;
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

// Named barrier among `nthreads` threads (ids 1..15 are free for kernels).
__device__ __forceinline__ void named_bar(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Launch with programmatic stream serialization: the kernel may start while
// the previous kernel in the stream drains; it must call griddepcontrol.wait
// (ptx::pdl_wait) before touching memory that kernel writes or reads.
// Programmatic dependent launch for every kernel launch of this library;
// SCHED_PDL=0 in the environment turns it off (plain stream-ordered launches).
inline bool pdl_enabled() {
  static const bool on = [] {
    const char *v = std::getenv("SCHED_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args &&...args) {
  if (!pdl_enabled()) {
    kernel<<<grid, block, smem, st>>>(std::forward<Args>(args)...);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
