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
  kEpiReduceScatter = 4,  // row-parallel, sequence-parallel output: push each finished bf16
                          // row only to the rank that owns the token and raise its row flag;
                          // the owner reduces (sched_sp_reduce_norm), no reduction here
};

// Token ownership of the sequence-parallel path: rank r owns the contiguous
// rows [r*T/world, (r+1)*T/world) (some ranks own none when T < world).
#ifdef __CUDACC__
__host__ __device__
#endif
inline int sp_row_owner(int t, int T, int world) {
  return (int)(((long long)(t + 1) * world - 1) / T);
}
#ifdef __CUDACC__
__host__ __device__
#endif
inline int sp_row_begin(int r, int T, int world) {
  return (int)((long long)r * T / world);
}

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
  int *status;    // 4 int32 words (code, site, int64 index of a bad index) or null
  // kEpiRopeKV only
  const int32_t *pos;    // [T] absolute positions
  const int32_t *slot;   // [T] page * page_size + offset, -1 = no cache write
  const float *cos_sin;  // [max_pos, 64, 2]
  __nv_bfloat16 *q_out;  // [T, Hq, 128]
  __nv_bfloat16 *k_cache, *v_cache;  // [pages, Hkv, page_size, 128]
  int Hq, Hkv, page_size;
  // kEpiAllReduce only: this rank's view of every rank's receive slab
  // [world][T][N] (bf16 partials) and flag array [world][tiles][TN/16] (u32,
  // zero between calls: the owner of a chunk resets its flags after use).
  // kEpiReduceScatter: the same slabs; the flag arrays are row flags
  // [world (source)][N/128][T] (u32, zero between calls: the owner of a row
  // resets them when it has reduced the row).
  int rank, world;
  __nv_bfloat16 *recv[kMaxWorld];
  uint32_t *flags[kMaxWorld];
  // optional per-CTA %globaltimer trace [grid][4]: entry, producer past the
  // dependency wait, last TMA issued, CTA done (nullptr: off)
  unsigned long long *trace;
  // kEpiRopeKV: pages of the KV cache; a token slot beyond them is reported
  // (kStatusBadIndex, site kSiteKvSlot) and not written. 0: unchecked.
  int kv_pages;
  // Gathered input (any epilogue; nullptr: none). Row t of x is read only
  // after x_ready[t] != 0: the owner of the row raises it with a
  // system-scope release once the row has landed in this rank's copy of x
  // (sched_sp_reduce_norm's all-gather push). Must be 16-byte aligned and
  // readable up to T rounded up to a multiple of 4.
  const uint32_t *x_ready;
  // kEpiAllReduce, low-latency exchange (ll_state != nullptr; decode sizes):
  // recv[j] is rank j's line buffer of two sets, each [world][T][N / 4]
  // 16-byte lines {bf16x2, epoch, bf16x2, epoch} (ll_set_lines lines per set),
  // and `flags` is unused. ll_state is this rank's [epoch, done] pair (u32,
  // zero before the first call): a call uses epoch + 1 and set (epoch + 1) & 1,
  // the last CTA to finish advances the epoch. Readers poll the lines until
  // both halves carry the call's epoch, so no fence, flag or reset is needed.
  uint32_t *ll_state;
  long long ll_set_lines;
  // Residual add + RMSNorm after the projection (kEpiStore, kEpiAllReduce;
  // norm_w != nullptr): once every n-tile of output row t is written to y,
  // the CTA that wrote the last one sets norm_res[t] += y[t] (bf16) and
  // norm_out[t] = rmsnorm(norm_res[t]) * norm_w, with the arithmetic and
  // reduction order of sched_add_rmsnorm (bit-identical results). row_cnt:
  // u32 [>= T] counters, zero between calls (the finishing CTA resets them).
  // Rows of norm_res / norm_out have N elements (contiguous); N <= 16384.
  __nv_bfloat16 *norm_res;
  const __nv_bfloat16 *norm_w;
  __nv_bfloat16 *norm_out;
  uint32_t *row_cnt;
  float norm_eps;
  // Low-latency exchange through NVLink multicast (NVLS; nullptr: off): this
  // rank's address of the multicast mapping of the line buffers, whose
  // local copy is recv[rank]. A line is then written once, as two 8-byte
  // multimem stores {bf16x2, epoch}, and the switch delivers it to every
  // rank's copy, instead of one store per rank.
  void *ll_mc;
};

extern "C" int sched_gemm_run(const GemmArgs *args, cudaStream_t stream);
// Schedule of a default-grid call: cluster size (0 = stream-K) and grid.
extern "C" void sched_gemm_plan(int T, int N, int K, int epi, int num_sms, int *cs, int *grid);
// The CTA-pair launch of a default-grid call: clusters (0: none), whole
// tiles, k-ranges per tile of the last wave.
extern "C" void sched_gemm_pair_plan(int T, int N, int K, int epi, long long ws_floats, int counters, int *np,
                                     int *whole, int *splits);
extern "C" long long sched_gemm_ws_floats(int T, int N, int K, int grid);

// ---------------------------------------------------------------------------
// Fixed-scratch entry point: sched_gemm_run without caller-provided scratch.
//
// No counterpart in the reference: it is for callers that may not allocate
// device memory at all (an embedding host whose allocator is off limits, a
// memory-capped sandbox, code that runs after the pool is sized). Instead of
// `ws` / `counters` it uses file-scope device arrays compiled into the
// module, so the call allocates nothing: no cudaMalloc or cudaFree and no
// caching allocator behind it.
//
//   * `ws`, `ws_floats`, `counters` and `counter_count` in *args are ignored;
//     every other field means what it means for sched_gemm_run.
//   * Scratch capacity is fixed: kFixedScratchWsFloats floats of stream-K
//     partial slices (16 MiB) and kFixedScratchCounters tile counters. A call
//     whose schedule needs more (sched_gemm_ws_floats(T, N, K, grid) above the
//     first, or more split tiles than the second) is refused with
//     kFixedScratchTooLarge before anything is launched; a smaller `grid`
//     needs less.
//   * The per-tile counters must be zero when a call starts. They start zero
//     (static storage) and each call that completes with a zero status word
//     leaves them zero again: the last CTA on a split tile resets its
//     counter. A call that reports a non-zero status (a bounded wait that
//     gave up) may leave them dirty: call sched_gemm_fixed_scratch_reset on
//     the stream before the next call on that device. The partial slices
//     need no initial value.
//   * The capacity check runs on the schedule the call will launch: a
//     default-grid call (grid <= 0) that runs cluster split-K uses no
//     scratch and is never refused for size, and one that runs the CTA-pair
//     kernel (prefill sizes) splits its last wave into k-ranges only as far
//     as their partials fit the fixed scratch (else it keeps tiles whole),
//     so it is never refused for size either.
//   * The scratch is one per device and shared by all calls on it: calls
//     that can overlap in time (different streams, or host threads on
//     unsynchronised streams) race on it and corrupt each other. Calls in
//     one stream are ordered and safe.
//   * The first call on each device looks up the arrays' device addresses
//     (cudaGetSymbolAddress, with that device current) and caches them;
//     make that first call before any stream capture begins. The stream must
//     belong to the current device.
//   * kEpiAllReduce and kEpiReduceScatter are refused
//     (kFixedScratchBadEpilogue): their peer receive buffers come from a
//     symmetric allocation.
// Returns 0, a sched_gemm_run code, or one of the codes below.
constexpr long long kFixedScratchWsFloats = 1ll << 22;
constexpr int kFixedScratchCounters = 1 << 14;
enum FixedScratchError : int {
  kFixedScratchTooLarge = -8,      // the call needs more scratch than the fixed capacity
  kFixedScratchLookupFailed = -9,  // no current device, or cudaGetSymbolAddress failed
  kFixedScratchBadEpilogue = -10,  // kEpiAllReduce, kEpiReduceScatter or a null args pointer
};
extern "C" int sched_gemm_run_fixed_scratch(const GemmArgs *args, cudaStream_t stream);
// Zeroes the fixed scratch's tile counters on the current device with one
// cudaMemsetAsync on `stream` (no allocation). Returns 0, or
// kFixedScratchLookupFailed / -4 (the memset was refused).
extern "C" int sched_gemm_fixed_scratch_reset(cudaStream_t stream);
