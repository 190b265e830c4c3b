// gemm_api.h -- host interface of the tcgen05 GEMM (csrc/kernels/gemm.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

enum GemmEpilogue : int {
  kEpiStore = 0,   // y[t, n] = acc
  kEpiSwiGLU = 1,  // y[t, j] = silu(gate) * up over interleaved 64-row gate/up blocks
  kEpiRopeKV = 2,  // fused QKV: rotate q/k heads, write q to q_out, k/v into the paged cache
  kEpiAllReduce = 3,  // row-parallel: push bf16 partial tiles to every rank over NVLink,
                      // then each rank sums the world's partials of the tiles it owns
};

constexpr int kMaxWorld = 8;

struct GemmArgs {
  const void *x;  // [T, K] bf16, row pitch ldx (elements)
  int ldx;
  const void *w;  // [N, K] bf16 row-major
  void *y;        // [T, ldy] bf16 (store / SwiGLU)
  int ldy;
  int T, N, K;
  int epi;
  int grid;       // CTAs (0: one per SM)
  int num_sms;
  float *ws;      // stream-K partial slices (see sched_gemm_ws_floats)
  long long ws_floats;
  uint32_t *counters;  // per-tile arrival counters, zero between calls
  int counter_count;
  int *status;
  // kEpiRopeKV only
  const int32_t *pos;    // [T] absolute positions
  const int32_t *slot;   // [T] page * page_size + offset, -1 = no cache write
  const float *cos_sin;  // [max_pos, 64, 2]
  __nv_bfloat16 *q_out;  // [T, Hq, 128]
  __nv_bfloat16 *k_cache, *v_cache;  // [pages, Hkv, page_size, 128]
  int Hq, Hkv, page_size;
  // kEpiAllReduce only: this rank's view of every rank's receive slab
  // [world][T][N] (bf16 partials) and flag array [world][tiles][TN/16] (u32,
  // zero between calls: the owner of a chunk resets its flags after use)
  int rank, world;
  __nv_bfloat16 *recv[kMaxWorld];
  uint32_t *flags[kMaxWorld];
};

extern "C" int sched_gemm_run(const GemmArgs *args, cudaStream_t stream);
extern "C" long long sched_gemm_ws_floats(int T, int N, int K, int grid);
