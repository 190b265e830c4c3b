// sp_api.h -- host interface of the sequence-parallel (SP) norm kernels
// (csrc/kernels/elementwise.cu), the middle of the tensor-parallel layer
//
//   row-parallel GEMM with kEpiReduceScatter   (o_proj / down_proj)
//     -> sched_sp_reduce_norm                  (reduce + residual + RMSNorm + all-gather push)
//     -> GEMM with GemmArgs::x_ready           (QKV / gate_up on the gathered rows)
//
// Rank r owns the token rows [r*T/world, (r+1)*T/world) (sp_row_begin).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemm_api.h"

struct SpNormArgs {
  const __nv_bfloat16 *slab;  // this rank's receive slab [world][T][H]: partials of its rows
  uint32_t *row_flags;        // this rank's row flags [world][H/128][T]; reset here after use
  __nv_bfloat16 *res;         // residual stream [T, H]: owned rows += reduced sum (bf16)
  const __nv_bfloat16 *w;     // RMSNorm weight [H]
  __nv_bfloat16 *delta;       // optional [T, H]: the reduced sum of the owned rows (nullptr: not kept)
  __nv_bfloat16 *gather[kMaxWorld];  // this rank's address of every rank's gathered rows [>= T][H]
  uint32_t *ready[kMaxWorld];        // this rank's address of every rank's row-ready flags [>= T]
  uint32_t *clear;            // this rank's ready flags of the other gather set (zeroed here)
  int clear_n;
  int T, H, rank, world;
  float eps;
  int *status;                // status words (kStatusPeerTimeout) or nullptr
};

// Reduce the world's partials of every owned row (rank order, fp32, rounded
// to bf16 once: the value the fused all-reduce produces), add it to the
// residual, RMSNorm the sum, and store the normed row into every rank's
// gather buffer, then raise the row's ready flag there (system-scope
// release). Also zeroes `clear` (the other gather set's flags, whose readers
// precede this kernel in stream order). Grid: one CTA per owned row (at
// least one). H: multiple of 128, at most 16384.
extern "C" int sched_sp_reduce_norm(const SpNormArgs *args, cudaStream_t stream);

// Wait (bounded) until ready[0..T) are all raised: orders a library kernel
// that reads the gathered rows (e.g. a row gather for sampling) after the
// all-gather. One CTA.
extern "C" int sched_sp_wait_rows(const uint32_t *ready, int T, int *status, cudaStream_t stream);
