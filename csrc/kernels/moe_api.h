// moe_api.h -- argument blocks of the MoE kernels (csrc/kernels/moe.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace moe {

constexpr int kMaxWorld = 8;
enum ExpertEpi : int { kExpSwiGLU = 0, kExpCombine = 1 };

struct DispatchArgs {
  const __nv_bfloat16 *x;  // [T, H] normalised token rows
  const int32_t *ids;      // [T, K]
  const float *wts;        // [T, K]
  int T, H, K, E, E_local, rank, world, capacity, rows_per_expert;
  // every rank's receive side, this process's addresses:
  uint8_t *slab[kMaxWorld];       // [E_local * rows_per_expert, H] fp8
  float *slab_scale[kMaxWorld];   // [E_local * rows_per_expert, H / 128]
  int32_t *slab_meta[kMaxWorld];  // [E_local * rows_per_expert, 4]: src rank, token, k, weight bits
  uint32_t *counter[kMaxWorld];   // [E_local] rows received per expert
  uint32_t *done[kMaxWorld];      // [1] sources finished
  uint32_t *local_done;           // this rank's count of finished dispatch CTAs
  __nv_bfloat16 *combine_local;   // this rank's combine buffer [T, K, H]
  uint32_t *dropped_step;         // this rank's assignments over capacity this layer
  uint32_t *dropped_total;        // ... accumulated (observability)
  int *status;
};

struct ExpertArgs {
  int E_local, N, K, rows_per_expert, n_tiles, t_tiles;
  const float *w_scale;  // [E_local, N / 128, K / 128]
  const float *x_scale;  // [K / 128, E_local * rows]: one row of token scales per K-block
  int ex_ld;             // x_scale row pitch (K / 128)
  // gate/up: wait for sources, then SwiGLU into act [E_local * rows, N / 2] bf16
  __nv_bfloat16 *act;
  uint32_t *counter;     // this rank's per-expert row counts
  uint32_t *done;        // this rank's finished-sources count
  uint32_t *rows_valid;  // [E_local] copy of the counts for the down GEMM
  uint32_t *tiles_done;  // CTA arrival counter (reset by the last CTA)
  int world, capacity;
  // down: combine rows back to their sources
  const int32_t *meta;   // [E_local * rows, 4]
  __nv_bfloat16 *combine[kMaxWorld];  // every rank's [T_src, K_top, H] buffer
  uint32_t *combine_cnt[kMaxWorld];   // every rank's received-row counter
  int k_top;
  int *status;
  // stream-K: partial slices [grid][2][TN * 128] fp32 and per-tile arrival
  // counters [E_local * n_tiles * t_tiles] (zero between calls)
  float *ws;
  uint32_t *tile_counters;
  int grid;  // persistent CTAs (0: one per SM)
  // optional per-CTA %globaltimer trace [grid][4]: entry, schedule known,
  // last TMA issued, epilogue done (nullptr: off)
  unsigned long long *trace;
};

}  // namespace moe

extern "C" int sched_moe_dispatch(const moe::DispatchArgs *a, cudaStream_t st);
extern "C" int sched_moe_expert_gemm(int epi, const void *w, const void *x, const moe::ExpertArgs *args,
                                     cudaStream_t st);
