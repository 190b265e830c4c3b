// gemm.cu -- bf16 GEMM on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
//   Y[T, N] = X[T, K] . W[N, K]^T          (Linear layer, weights row-major)
//
// Decode-first design ("swap-AB"): the MMA's M dimension runs over 128 rows
// of the weight (output features) and its N dimension over a tile of TN
// tokens (16..256). A decode step has few tokens and many weight rows, so the
// weight stream -- the HBM-bound part -- always fills the 128-row MMA, and
// the token count only sets the (cheap) N width. Prefill uses TN = 256.
//
// One CTA = 6 warps:
//   warp 0  TMA producer: one elected thread streams W and X K-blocks (64
//           elements = one 128-byte swizzle atom) into an STAGES-deep ring;
//   warp 1  MMA issuer: one thread issues 4 x tcgen05.mma (K = 16 each) per
//           stage into a TMEM accumulator [128 lanes x TN columns], and
//           tcgen05.commit frees the stage when those MMAs retire;
//   warps 2-5 epilogue: tcgen05.ld the accumulator, stage 16-token slabs in
//           shared memory, and write coalesced rows.
//
// Split-K (decode): when the (row-tile x token-tile) grid cannot fill the
// 148 SMs, K is split S ways. Every split stores its fp32 partial tile into
// its own slice of a workspace [S][T_pad][N]; the last split to finish a tile
// (per-tile arrival counter) sums the S slices in split order -- a fixed
// order, so results are bit-reproducible run to run -- applies the epilogue,
// writes bf16 and resets the tile's counter to zero (counters stay zero
// between calls; the partial slices need no clearing because every split
// rewrites its slice). Calls sharing one workspace must not run concurrently.
//
// Epilogues: plain store, or SwiGLU over an interleaved gate/up weight whose
// 128-row tile holds 64 gate rows followed by the 64 matching up rows
// (out[t, j] = silu(gate) * up), which fuses the MLP activation into the
// gate_up projection.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <stdexcept>

#include "common.cuh"
#include "sched/ptx.cuh"
#include "tmap.h"

namespace gemm {

constexpr int BM = 128;  // weight rows per tile (MMA M)
constexpr int BK = 64;   // K elements per stage (128 bytes of bf16)
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;
constexpr int kSlab = 16;  // tokens per epilogue slab
constexpr int kSlabPitch = BM + 4;

enum Epi : int { kEpiStore = 0, kEpiSwiGLU = 1 };

template <int TN>
struct Cfg {
  static constexpr int W_BYTES = BM * BK * 2;
  static constexpr int X_BYTES = TN * BK * 2;
  static constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
  static constexpr int STAGES = TN >= 256 ? 4 : (TN >= 128 ? 3 : (TN >= 64 ? 4 : 5));
  static constexpr int TMEM_COLS = TN < 32 ? 32 : TN;
  static constexpr int SLAB_BYTES = kSlab * kSlabPitch * 4;
  static constexpr int SMEM = 1024 /*align*/ + STAGES * STAGE_BYTES + SLAB_BYTES + 256;
};

struct Params {
  __nv_bfloat16 *y;
  int T, N, K, ldy;
  int n_tiles, t_tiles, splits, kb_per_split;
  float *ws;           // [splits, T_pad, N] fp32 partial tiles (split > 1 only)
  uint32_t *counters;  // [n_tiles * t_tiles], zero between calls
  int *status;
};

template <int TN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_swapab_kernel(const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmX, Params p) {
  using C = Cfg<TN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *stage_mem = base;
  float *slab = reinterpret_cast<float *>(base + C::STAGES * C::STAGE_BYTES);
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + C::STAGES * C::STAGE_BYTES + C::SLAB_BYTES);
  uint64_t *full = bars;
  uint64_t *empty = bars + C::STAGES;
  uint64_t *accum = bars + 2 * C::STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * C::STAGES + 1);
  __shared__ int last_flag;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  // unit -> (split, n_tile, t_tile); token tiles innermost so neighbouring
  // CTAs reuse the same weight tile from L2 during prefill.
  int unit = blockIdx.x;
  const int t_tile = unit % p.t_tiles;
  unit /= p.t_tiles;
  const int n_tile = unit % p.n_tiles;
  const int split = unit / p.n_tiles;
  const int kb_total = p.K / BK;
  const int kb_begin = split * p.kb_per_split;
  const int kb_end = min(kb_total, kb_begin + p.kb_per_split);
  const int nkb = kb_end - kb_begin;

  if (warp == 0) {
    ptx::tmem_alloc(tmem_slot, C::TMEM_COLS);
    ptx::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < C::STAGES; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    ptx::mbar_init(accum, 1);
    ptx::fence_mbar_init();
  }
  if (threadIdx.x == 64) {
    ptx::prefetch_tmap(&tmW);
    ptx::prefetch_tmap(&tmX);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (ptx::elect_one()) {
      for (int i = 0; i < nkb; ++i) {
        const int s = i % C::STAGES;
        const uint32_t ph = (i / C::STAGES) & 1;
        if (!ptx::mbar_wait(&empty[s], ph ^ 1, kWaitBudgetNs)) {
          report_status(p.status, kStatusMmaTimeout);
          break;
        }
        uint8_t *st = stage_mem + s * C::STAGE_BYTES;
        ptx::mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
        const int kc = (kb_begin + i) * BK;
        ptx::tma_load_2d(st, &tmW, &full[s], kc, n_tile * BM);
        ptx::tma_load_2d(st + C::W_BYTES, &tmX, &full[s], kc, t_tile * TN);
      }
    }
  } else if (warp == 1) {
    if (ptx::elect_one()) {
      constexpr uint32_t idesc = ptx::idesc_f16(BM, TN, /*bf16*/ 1, false, false);
      bool ok = true;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % C::STAGES;
        const uint32_t ph = (i / C::STAGES) & 1;
        if (!ptx::mbar_wait(&full[s], ph, kWaitBudgetNs)) {
          report_status(p.status, kStatusTmaTimeout);
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        uint8_t *st = stage_mem + s * C::STAGE_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          uint64_t a = ptx::smem_desc(st + kk * 32, 16, 1024, ptx::kLayoutSW128);
          uint64_t b = ptx::smem_desc(st + C::W_BYTES + kk * 32, 16, 1024, ptx::kLayoutSW128);
          ptx::mma_f16_ss(tmem, a, b, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        }
        ptx::mma_commit(&empty[s]);
      }
      (void)ok;
      ptx::mma_commit(accum);  // fires once all issued MMAs retire (immediately if none)
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int et = threadIdx.x - 64;  // 0..127
    const int q = warp & 3;           // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;    // accumulator row = weight row within the tile
    const bool waited = ptx::mbar_wait(accum, 0, kWaitBudgetNs);
    if (!waited) report_status(p.status, kStatusEpilogueTimeout);
    ptx::tc_fence_after();
    const int t0 = t_tile * TN;
    const int n0 = n_tile * BM;
    const bool direct = (p.splits == 1);
    for (int c = 0; c < TN / kSlab; ++c) {
      if (t0 + c * kSlab >= p.T) break;
      uint32_t r[16];
      ptx::tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + c * kSlab, r);
      ptx::tmem_ld_wait();
      if (nkb == 0 || !waited) {
#pragma unroll
        for (int j = 0; j < 16; ++j) r[j] = 0u;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) slab[j * kSlabPitch + row] = __uint_as_float(r[j]);
      named_bar(1, kEpiThreads);
      // 16 tokens x 128 rows: each thread handles 16 consecutive values of one token.
      const int tj = et / 8;          // token within slab
      const int col = (et % 8) * 16;  // first row (feature) of this thread's run
      const int t = t0 + c * kSlab + tj;
      if (t < p.T) {
        const float *src = slab + tj * kSlabPitch + col;
        if (direct) {
          if (EPI == kEpiStore) {
            uint4 o0, o1;
            o0.x = pack_bf16x2(src[0], src[1]);
            o0.y = pack_bf16x2(src[2], src[3]);
            o0.z = pack_bf16x2(src[4], src[5]);
            o0.w = pack_bf16x2(src[6], src[7]);
            o1.x = pack_bf16x2(src[8], src[9]);
            o1.y = pack_bf16x2(src[10], src[11]);
            o1.z = pack_bf16x2(src[12], src[13]);
            o1.w = pack_bf16x2(src[14], src[15]);
            uint4 *dst = reinterpret_cast<uint4 *>(p.y + (size_t)t * p.ldy + n0 + col);
            dst[0] = o0;
            dst[1] = o1;
          } else if (col < 64) {
            // SwiGLU: rows [0,64) are gate, [64,128) the matching up rows.
            const float *up = src + 64;
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = silu(src[j]) * up[j];
            uint4 o0, o1;
            o0.x = pack_bf16x2(v[0], v[1]);
            o0.y = pack_bf16x2(v[2], v[3]);
            o0.z = pack_bf16x2(v[4], v[5]);
            o0.w = pack_bf16x2(v[6], v[7]);
            o1.x = pack_bf16x2(v[8], v[9]);
            o1.y = pack_bf16x2(v[10], v[11]);
            o1.z = pack_bf16x2(v[12], v[13]);
            o1.w = pack_bf16x2(v[14], v[15]);
            uint4 *dst = reinterpret_cast<uint4 *>(p.y + (size_t)t * p.ldy + n_tile * 64 + col);
            dst[0] = o0;
            dst[1] = o1;
          }
        } else {
          const size_t t_pad = (size_t)p.t_tiles * TN;
          float4 *dst = reinterpret_cast<float4 *>(p.ws + ((size_t)split * t_pad + t) * p.N + n0 + col);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            __stcg(dst + j, make_float4(src[4 * j], src[4 * j + 1], src[4 * j + 2], src[4 * j + 3]));
        }
      }
      named_bar(1, kEpiThreads);
    }
    if (!direct) {
      // Arrival: the last split of this tile finishes it.
      if (et == 0) {
        __threadfence();
        uint32_t prev = atomicAdd(&p.counters[n_tile * p.t_tiles + t_tile], 1u);
        last_flag = (prev == (uint32_t)(p.splits - 1)) ? 1 : 0;
      }
      named_bar(1, kEpiThreads);
      if (last_flag) {
        __threadfence();
        const int tmax = min(TN, p.T - t0);
        const size_t slice = (size_t)p.t_tiles * TN * p.N;
        // 128 threads sweep the [tmax x 128] tile, 8 features per thread-step;
        // SwiGLU threads own 8 gate rows and read the matching 8 up rows.
        for (int idx = et; idx < tmax * (BM / 8); idx += kEpiThreads) {
          const int tj = idx / (BM / 8);
          const int col = (idx % (BM / 8)) * 8;
          if (EPI == kEpiSwiGLU && col >= 64) continue;
          const int t = t0 + tj;
          const float *src = p.ws + (size_t)t * p.N + n0 + col;
          float a[8], u[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) a[j] = u[j] = 0.f;
          for (int sp = 0; sp < p.splits; ++sp) {
            const float4 *s4 = reinterpret_cast<const float4 *>(src + sp * slice);
            const float4 x0 = __ldcg(s4), x1 = __ldcg(s4 + 1);
            a[0] += x0.x; a[1] += x0.y; a[2] += x0.z; a[3] += x0.w;
            a[4] += x1.x; a[5] += x1.y; a[6] += x1.z; a[7] += x1.w;
            if (EPI == kEpiSwiGLU) {
              const float4 y0 = __ldcg(s4 + 16), y1 = __ldcg(s4 + 17);  // +64 floats: up rows
              u[0] += y0.x; u[1] += y0.y; u[2] += y0.z; u[3] += y0.w;
              u[4] += y1.x; u[5] += y1.y; u[6] += y1.z; u[7] += y1.w;
            }
          }
          uint4 o;
          if (EPI == kEpiStore) {
            o.x = pack_bf16x2(a[0], a[1]);
            o.y = pack_bf16x2(a[2], a[3]);
            o.z = pack_bf16x2(a[4], a[5]);
            o.w = pack_bf16x2(a[6], a[7]);
            *reinterpret_cast<uint4 *>(p.y + (size_t)t * p.ldy + n0 + col) = o;
          } else {
            o.x = pack_bf16x2(silu(a[0]) * u[0], silu(a[1]) * u[1]);
            o.y = pack_bf16x2(silu(a[2]) * u[2], silu(a[3]) * u[3]);
            o.z = pack_bf16x2(silu(a[4]) * u[4], silu(a[5]) * u[5]);
            o.w = pack_bf16x2(silu(a[6]) * u[6], silu(a[7]) * u[7]);
            *reinterpret_cast<uint4 *>(p.y + (size_t)t * p.ldy + n_tile * 64 + col) = o;
          }
        }
        if (et == 0) p.counters[n_tile * p.t_tiles + t_tile] = 0u;
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) ptx::tmem_dealloc(tmem, C::TMEM_COLS);
}

template <int TN, int EPI>
static void launch_tn(const CUtensorMap &tw, const CUtensorMap &tx, const Params &p, int grid,
                      cudaStream_t stream) {
  using C = Cfg<TN>;
  auto kern = gemm_swapab_kernel<TN, EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    attr_set = true;
  }
  kern<<<grid, kThreads, C::SMEM, stream>>>(tw, tx, p);
}

template <int EPI>
static void dispatch(int tn, const CUtensorMap &tw, const CUtensorMap &tx, const Params &p,
                     int grid, cudaStream_t stream) {
  switch (tn) {
    case 16: launch_tn<16, EPI>(tw, tx, p, grid, stream); break;
    case 32: launch_tn<32, EPI>(tw, tx, p, grid, stream); break;
    case 64: launch_tn<64, EPI>(tw, tx, p, grid, stream); break;
    case 128: launch_tn<128, EPI>(tw, tx, p, grid, stream); break;
    default: launch_tn<256, EPI>(tw, tx, p, grid, stream); break;
  }
}

}  // namespace gemm

// Token-tile width for T tokens.
static int pick_tn(int T) {
  if (T <= 16) return 16;
  if (T <= 32) return 32;
  if (T <= 64) return 64;
  if (T <= 128) return 128;
  return 256;
}

extern "C" int sched_gemm_split_count(int T, int N, int K, int num_sms) {
  const int tn = pick_tn(T);
  const int units = (N / gemm::BM) * ((T + tn - 1) / tn);
  const int kb = K / gemm::BK;
  const int target = 2 * num_sms;
  if (units >= num_sms) return 1;
  int s = (target + units - 1) / units;
  s = std::min(s, std::max(1, kb / 4));
  return std::max(1, s);
}

// Host launcher. Returns 0 on success, a negative value on a bad argument.
//   x  [T, K] bf16 row-major (pitch ldx), w [N, K] bf16 row-major,
//   y  [T, ldy] bf16; epi 0: ldy >= N, epi 1 (SwiGLU): writes N/2 columns.
//   ws/counters: split-K workspace ([splits x T_pad x N] fp32, and
//   n_tiles*t_tiles u32 counters that must be zero) -- required when splits > 1.
extern "C" int sched_gemm_bf16(const void *x, int ldx, const void *w, void *y, int ldy, int T,
                               int N, int K, int epi, int splits, float *ws, uint32_t *counters,
                               int *status, cudaStream_t stream) {
  if (T <= 0) return 0;
  if (N % gemm::BM != 0 || K % gemm::BK != 0) return -1;
  if (splits > 1 && (ws == nullptr || counters == nullptr)) return -2;
  const int tn = pick_tn(T);
  gemm::Params p;
  p.y = static_cast<__nv_bfloat16 *>(y);
  p.T = T;
  p.N = N;
  p.K = K;
  p.ldy = ldy;
  p.n_tiles = N / gemm::BM;
  p.t_tiles = (T + tn - 1) / tn;
  const int kb = K / gemm::BK;
  splits = std::max(1, std::min(splits, kb));
  p.kb_per_split = (kb + splits - 1) / splits;
  p.splits = (kb + p.kb_per_split - 1) / p.kb_per_split;
  p.ws = ws;
  p.counters = counters;
  p.status = status;
  try {
    CUtensorMap tw = tmap::make_2d(w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, K, gemm::BM,
                                   gemm::BK, CU_TENSOR_MAP_SWIZZLE_128B);
    CUtensorMap tx = tmap::make_2d(x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, K, ldx, tn, gemm::BK,
                                   CU_TENSOR_MAP_SWIZZLE_128B);
    const int grid = p.n_tiles * p.t_tiles * p.splits;
    if (epi == gemm::kEpiSwiGLU)
      gemm::dispatch<gemm::kEpiSwiGLU>(tn, tw, tx, p, grid, stream);
    else
      gemm::dispatch<gemm::kEpiStore>(tn, tw, tx, p, grid, stream);
  } catch (const std::exception &) {
    return -3;
  }
  return (int)cudaPeekAtLastError() == 0 ? 0 : -4;
}
