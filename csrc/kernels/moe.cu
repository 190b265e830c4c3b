// moe.cu -- mixture-of-experts layer for expert parallelism over NVLink.
//
// Per MoE layer and rank (experts are split across ranks, E_local each):
//   1. router_topk    softmax top-k routing of the local tokens;
//   2. dispatch       every (token, k) assignment quantises the token row to
//                     fp8 e4m3 with one fp32 scale per 128 columns and stores
//                     it straight into the owning rank's receive slab over
//                     NVLink (P2P stores); its slot comes from a system-scope
//                     atomic on the owner's per-expert counter, which is also
//                     where the capacity lever acts (slots >= capacity drop
//                     the assignment: GShard/Switch capacity, E2). Each
//                     source then raises one "done" count per owner;
//   3. expert GEMMs   fp8 x fp8 on tcgen05 (kind::f8f6f4) with 128x128 weight
//                     block scales and 1x128 activation scales, promoted per
//                     128-K block: each block's MMAs land in one of two TMEM
//                     partials and the epilogue warps fold
//                     partial * s_w * s_x into register accumulators while
//                     the next block's MMAs run. The gate/up GEMM waits
//                     (bounded) for every source's done count before reading
//                     rows and finishes with SwiGLU; the down GEMM's epilogue
//                     IS the combine: each finished row, scaled by its
//                     routing weight, is stored back into the source rank's
//                     combine buffer over NVLink and counted there;
//   4. combine_norm   the source waits (bounded) for all its rows, sums the k
//                     contributions, adds the residual and applies RMSNorm
//                     (the next sub-block's input) in one pass.
// Counters are reset by their single consumer before any producer can reuse
// them, so no per-step memset is needed.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>

#include "common.cuh"
#include "sched/ptx.cuh"
#include "tmap.h"
#include "moe_api.h"

namespace moe {

constexpr int kMaxTopK = 8;
constexpr int QB = 128;  // quantisation block (columns)

// ---------------------------------------------------------------- routing
// One CTA per token, one warp per expert: logits over E experts (bf16 router
// weight [E, H]), top-k by value, weights = softmax over the selected logits
// (Mixtral). Every warp's loads are independent, so the dot products overlap.
__global__ void router_topk_kernel(const __nv_bfloat16 *__restrict__ x, const __nv_bfloat16 *__restrict__ wr,
                                   int T, int H, int E, int K, int32_t *__restrict__ ids,
                                   float *__restrict__ wts) {
  __shared__ float logit[32];
  const int t = blockIdx.x, e = threadIdx.x / 32, lane = threadIdx.x % 32;
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const __nv_bfloat16 *row = x + (size_t)t * H;
  const __nv_bfloat16 *w = wr + (size_t)e * H;
  float s = 0.f;
#pragma unroll 4
  for (int c = lane * 8; c < H; c += 256) {
    const uint4 a = *reinterpret_cast<const uint4 *>(row + c);
    const uint4 b = __ldg(reinterpret_cast<const uint4 *>(w + c));
    const __nv_bfloat16 *ae = reinterpret_cast<const __nv_bfloat16 *>(&a);
    const __nv_bfloat16 *be = reinterpret_cast<const __nv_bfloat16 *>(&b);
#pragma unroll
    for (int j = 0; j < 8; ++j) s += __bfloat162float(ae[j]) * __bfloat162float(be[j]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) logit[e] = s;
  __syncwarp();
  __syncthreads();
  if (threadIdx.x == 0) {
    int sel[kMaxTopK];
    float val[kMaxTopK];
    unsigned used = 0;
    for (int k = 0; k < K; ++k) {
      int best = -1;
      for (int j = 0; j < E; ++j)
        if (!(used >> j & 1u) && (best < 0 || logit[j] > logit[best])) best = j;
      used |= 1u << best;
      sel[k] = best;
      val[k] = logit[best];
    }
    float m = val[0], den = 0.f;
    for (int k = 0; k < K; ++k) den += __expf(val[k] - m);
    for (int k = 0; k < K; ++k) {
      ids[t * K + k] = sel[k];
      wts[t * K + k] = __expf(val[k] - m) / den;
    }
  }
}

// ---------------------------------------------------------------- dispatch
// One CTA (128 threads) per token: its K slots are claimed in parallel, the
// row is quantised once (one fp32 scale per 128 columns) and stored to every
// destination slab.
__global__ void __launch_bounds__(128) dispatch_kernel(const DispatchArgs a) {
  const int t = blockIdx.x;
  __shared__ int slot_s[kMaxTopK];
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  if (t < a.T) {
    if (threadIdx.x < a.K) {
      const int k = threadIdx.x;
      const int e = a.ids[t * a.K + k];
      const int owner = e / a.E_local, le = e % a.E_local;
      const uint32_t s = atomicAdd_system(a.counter[owner] + le, 1u);
      slot_s[k] = (int)s < a.capacity ? (int)s : -1;
      if (slot_s[k] < 0) {
        atomicAdd(a.dropped_step, 1u);
        if (a.dropped_total) atomicAdd(a.dropped_total, 1u);
      }
    }
    __syncwarp();
    __syncthreads();
    const __nv_bfloat16 *src = a.x + (size_t)t * a.H;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    for (int blk = warp; blk < a.H / QB; blk += 4) {
      const uint2 u = *reinterpret_cast<const uint2 *>(src + blk * QB + lane * 4);
      const __nv_bfloat16 *v = reinterpret_cast<const __nv_bfloat16 *>(&u);
      float f[4], m = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        f[j] = __bfloat162float(v[j]);
        m = fmaxf(m, fabsf(f[j]));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float scale = m > 0.f ? m / 448.f : 1.f;
      const float inv = 1.f / scale;
      uint32_t packed = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_fp8_e4m3 q(f[j] * inv);
        packed |= (uint32_t)(*reinterpret_cast<const uint8_t *>(&q)) << (8 * j);
      }
      for (int k = 0; k < a.K; ++k) {
        const int slot = slot_s[k];
        if (slot < 0) continue;
        const int e = a.ids[t * a.K + k];
        const int owner = e / a.E_local, le = e % a.E_local;
        const size_t row = (size_t)le * a.rows_per_expert + slot;
        *reinterpret_cast<uint32_t *>(a.slab[owner] + row * a.H + blk * QB + lane * 4) = packed;
        if (lane == 0) a.slab_scale[owner][(size_t)blk * a.E_local * a.rows_per_expert + row] = scale;
      }
    }
    if (threadIdx.x < a.K) {
      const int k = threadIdx.x;
      const int e = a.ids[t * a.K + k];
      const int owner = e / a.E_local, le = e % a.E_local;
      if (slot_s[k] >= 0) {
        const size_t row = (size_t)le * a.rows_per_expert + slot_s[k];
        *reinterpret_cast<int4 *>(a.slab_meta[owner] + row * 4) =
            make_int4(a.rank, t, k, __float_as_int(a.wts[t * a.K + k]));
      }
    }
    // dropped assignments contribute zero rows to the local combine buffer
    for (int k = 0; k < a.K; ++k) {
      if (slot_s[k] >= 0) continue;
      __nv_bfloat16 *c = a.combine_local + ((size_t)t * a.K + k) * a.H;
      for (int col = threadIdx.x * 8; col < a.H; col += 128 * 8)
        *reinterpret_cast<uint4 *>(c + col) = make_uint4(0, 0, 0, 0);
    }
  }
  // the last dispatch CTA of this rank announces completion to every owner
  // (a rank with no tokens launches one CTA that only announces)
  ptx::fence_acq_rel_sys();
  __syncwarp();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t fin = atomicAdd(a.local_done, 1u);
    if (fin == gridDim.x - 1) {
      *a.local_done = 0u;
      ptx::fence_acq_rel_sys();
      for (int r = 0; r < a.world; ++r) atomicAdd_system(a.done[r], 1u);
    }
  }
}

// ---------------------------------------------------------------- fp8 expert GEMM
// Persistent stream-K over the ACTIVE tiles only. How many rows each expert
// received is known on the device alone, so every CTA derives the same
// schedule from the row counts: tiles (expert, n-tile, token-tile) with
// token tiles fastest (CTAs running together share each weight tile through
// L2), units = tiles x K-blocks split evenly over the grid. A tile cut
// between CTAs is reduced by its last-arriving CTA from per-CTA fp32 slices
// in a fixed order (deterministic), exactly like the dense GEMM.
constexpr int BM = 128;
constexpr int BK = 128;  // fp8 elements per stage = 128 bytes
constexpr int TN = 64;   // rows (tokens) per tile
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter, each on half of the tokens
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kThreads = 64 + kEpiThreads;
constexpr int HALF = TN / 2;
constexpr int NP = 8;  // TMEM partial buffers (per-K-block MMA results)
constexpr int W_BYTES = BM * BK;
constexpr int X_BYTES = TN * BK;
constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
constexpr int STAGES = 8;
constexpr int UP_PITCH = TN + 1;                // [64 up rows][TN tokens] fp32, conflict-free
constexpr int UP_BYTES = (BM / 2) * UP_PITCH * 4;
constexpr int kMaxExperts = 32;
constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + UP_BYTES + 1024;

struct Sched {
  int tprefix[kMaxExperts + 1];  // active-tile prefix over experts
  int ttc[kMaxExperts];          // token tiles of each expert
  int rows[kMaxExperts];
  long long units;
  int kb;
};

struct Seg {
  int tile, kb0, kb1, seg, nsegs;
};

// Units go to the first G = min(grid, units) CTAs, so every one of them gets
// at least one unit and a tile's segments are exactly CTAs c0..c1.
__device__ __forceinline__ long long eff_grid(const Sched &s) {
  return s.units < (long long)gridDim.x ? s.units : (long long)gridDim.x;
}
__device__ __forceinline__ long long unit_begin(const Sched &s, int c) {
  const long long G = eff_grid(s);
  return c >= G ? s.units : (long long)c * s.units / G;
}
__device__ __forceinline__ int cta_of_unit(const Sched &s, long long u) {
  return (int)(((u + 1) * eff_grid(s) - 1) / s.units);
}
__device__ __forceinline__ bool segment(const Sched &s, int c, int k, Seg &g) {
  const long long b = unit_begin(s, c), e = unit_begin(s, c + 1);
  if (b >= e) return false;
  const int tile = (int)(b / s.kb) + k;
  const long long tb = (long long)tile * s.kb, te = tb + s.kb;
  if (tb >= e) return false;
  g.tile = tile;
  g.kb0 = (int)(max(b, tb) - tb);
  g.kb1 = (int)(min(e, te) - tb);
  const int c0 = cta_of_unit(s, tb), c1 = cta_of_unit(s, te - 1);
  g.seg = c - c0;
  g.nsegs = c1 - c0 + 1;
  return true;
}
__device__ __forceinline__ void tile_coords(const Sched &s, int E_local, int tile, int &ex, int &nt, int &tt) {
  ex = 0;
  while (ex + 1 < E_local && tile >= s.tprefix[ex + 1]) ++ex;
  const int j = tile - s.tprefix[ex];
  nt = j / s.ttc[ex];
  tt = j % s.ttc[ex];
}

// gate/up: the last CTA publishes the row counts for the down GEMM and
// clears the receive counters (every CTA read them at its start).
__device__ __forceinline__ void finish_gate_up(const ExpertArgs &a) {
  __threadfence();
  const uint32_t fin = atomicAdd(a.tiles_done, 1u);
  if (fin == gridDim.x - 1) {
    for (int e = 0; e < a.E_local; ++e) {
      a.rows_valid[e] = min((uint32_t)a.capacity, a.counter[e]);
      a.counter[e] = 0u;
    }
    *a.done = 0u;
    *a.tiles_done = 0u;
    __threadfence_system();
  }
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    expert_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                       const ExpertArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float *up_sm = reinterpret_cast<float *>(base + STAGES * STAGE_BYTES);  // [64][UP_PITCH]
  uint64_t *bars = reinterpret_cast<uint64_t *>(up_sm + (BM / 2) * UP_PITCH);
  uint64_t *full = bars, *empty = bars + STAGES;
  uint64_t *p_full = bars + 2 * STAGES, *p_empty = bars + 2 * STAGES + NP;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 2 * NP);
  volatile int *last_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  __shared__ Sched sch;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int c = blockIdx.x;
  const size_t x_rows = (size_t)a.E_local * a.rows_per_expert;  // x_scale is [K / 128][x_rows]

  ptx::pdl_launch_dependents();
  if (warp == 0) {
    ptx::tmem_alloc(tmem_slot, NP * TN);
    ptx::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < NP; ++i) {
      ptx::mbar_init(&p_full[i], 1);
      ptx::mbar_init(&p_empty[i], kEpiThreads);
    }
    ptx::fence_mbar_init();
  }
  if (threadIdx.x == 64) {
    ptx::prefetch_tmap(&tmW);
    ptx::prefetch_tmap(&tmX);
  }
  // the schedule: rows per expert (gate/up waits for every source first)
  if (threadIdx.x == 0) {
    if (a.trace) a.trace[c * 4] = ptx::globaltimer_ns();
    ptx::pdl_wait();
    if (EPI == kExpSwiGLU) {
      bool ok = ptx::ld_acquire_sys(a.done) >= (uint32_t)a.world;
      if (!ok) {
        const uint64_t t0 = ptx::globaltimer_ns();
        while (!ok && ptx::globaltimer_ns() - t0 < kWaitBudgetNs) ok = ptx::ld_acquire_sys(a.done) >= (uint32_t)a.world;
        if (!ok) report_status(a.status, kStatusPeerTimeout);
      }
    }
    int acc = 0;
    for (int e = 0; e < a.E_local; ++e) {
      const uint32_t n = EPI == kExpSwiGLU ? ptx::ld_acquire_sys(a.counter + e) : __ldcg(a.rows_valid + e);
      const int rows = min(min((int)n, a.capacity), a.rows_per_expert);
      sch.rows[e] = rows;
      sch.ttc[e] = (rows + TN - 1) / TN;
      sch.tprefix[e] = acc;
      acc += sch.ttc[e] * a.n_tiles;
    }
    sch.tprefix[a.E_local] = acc;
    sch.kb = a.K / BK;
    sch.units = (long long)acc * sch.kb;
  }
  ptx::tc_fence_before();
  __syncwarp();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (a.trace && threadIdx.x == 0) a.trace[c * 4 + 1] = ptx::globaltimer_ns();

  if (sch.units > 0 && warp == 0) {
    // ============================================================ producer
    if (ptx::elect_one()) {
      // slab rows arrived through peers' generic stores; TMA reads them
      ptx::fence_proxy_async_global();
      Seg g;
      int i = 0;
      bool ok = true;
      for (int k = 0; ok && segment(sch, c, k, g); ++k) {
        int ex, nt, tt;
        tile_coords(sch, a.E_local, g.tile, ex, nt, tt);
        for (int kb = g.kb0; kb < g.kb1; ++kb, ++i) {
          const int st = i % STAGES;
          if (!ptx::mbar_wait(&empty[st], ((i / STAGES) & 1) ^ 1)) {
            report_status(a.status, kStatusMmaTimeout);
            ok = false;
            break;
          }
          uint8_t *sm = base + st * STAGE_BYTES;
          ptx::mbar_arrive_expect_tx(&full[st], STAGE_BYTES);
          ptx::tma_load_2d(sm, &tmW, &full[st], kb * BK, ex * a.N + nt * BM);
          ptx::tma_load_2d(sm + W_BYTES, &tmX, &full[st], kb * BK, ex * a.rows_per_expert + tt * TN);
        }
      }
      if (a.trace) a.trace[c * 4 + 2] = ptx::globaltimer_ns();
    }
  } else if (sch.units > 0 && warp == 1) {
    // ============================================================ MMA
    if (ptx::elect_one()) {
      constexpr uint32_t idesc = ptx::idesc_e4m3(BM, TN);
      Seg g;
      int i = 0;
      bool ok = true;
      for (int k = 0; ok && segment(sch, c, k, g); ++k) {
        for (int kb = g.kb0; kb < g.kb1; ++kb, ++i) {
          const int st = i % STAGES, pb = i % NP;
          if (!ptx::mbar_wait(&full[st], (i / STAGES) & 1) ||
              !ptx::mbar_wait(&p_empty[pb], ((i / NP) & 1) ^ 1)) {
            report_status(a.status, kStatusTmaTimeout);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          uint8_t *sm = base + st * STAGE_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            const uint64_t da = ptx::smem_desc(sm + kk * 32, 16, 1024, ptx::kLayoutSW128);
            const uint64_t db = ptx::smem_desc(sm + W_BYTES + kk * 32, 16, 1024, ptx::kLayoutSW128);
            ptx::mma_f8_ss(tmem + pb * TN, da, db, idesc, kk > 0 ? 1u : 0u);
          }
          ptx::mma_commit(&empty[st]);
          ptx::mma_commit(&p_full[pb]);
        }
      }
    }
  } else if (sch.units > 0 && warp >= 2) {
    // ============================================================ promotion + epilogue
    // acc[t] += partial[row][t] * s_w[kb] * s_x[kb][t]; warp pair (q, half)
    // covers TMEM lanes 32q.. and token columns half*32..
    const int q = warp & 3, hf = (warp - 2) / 4, row = q * 32 + lane, et = threadIdx.x - 64;
    Seg g;
    int i = 0;
    bool ok = true;
    for (int k = 0; segment(sch, c, k, g); ++k) {
      int ex, nt, tt;
      tile_coords(sch, a.E_local, g.tile, ex, nt, tt);
      const int r0 = ex * a.rows_per_expert + tt * TN;
      const float *sw = a.w_scale + ((size_t)ex * a.n_tiles + nt) * sch.kb;
      float acc[HALF];
#pragma unroll
      for (int j = 0; j < HALF; ++j) acc[j] = 0.f;
      for (int kb = g.kb0; kb < g.kb1; ++kb, ++i) {
        const int pb = i % NP;
        // this K-block's activation scales of our 32 tokens (warp-uniform: broadcast loads)
        const float4 *xs4 = reinterpret_cast<const float4 *>(a.x_scale + (size_t)kb * x_rows + r0 + hf * HALF);
        float s[HALF];
        const float swk = __ldg(sw + kb);
#pragma unroll
        for (int j = 0; j < HALF / 4; ++j) {
          const float4 v = __ldg(xs4 + j);
          s[4 * j] = v.x * swk;
          s[4 * j + 1] = v.y * swk;
          s[4 * j + 2] = v.z * swk;
          s[4 * j + 3] = v.w * swk;
        }
        if (ok && !ptx::mbar_wait(&p_full[pb], (i / NP) & 1)) {
          report_status(a.status, kStatusEpilogueTimeout);
          ok = false;
        }
        ptx::tc_fence_after();
        uint32_t r0v[16], r1v[16];
        const uint32_t taddr = tmem + pb * TN + hf * HALF + ((uint32_t)(q * 32) << 16);
        ptx::tmem_ld16(taddr, r0v);
        ptx::tmem_ld16(taddr + 16, r1v);
        ptx::tmem_ld_wait();
        ptx::tc_fence_before();
        ptx::mbar_arrive(&p_empty[pb]);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          acc[j] = fmaf(__uint_as_float(r0v[j]), s[j], acc[j]);
          acc[16 + j] = fmaf(__uint_as_float(r1v[j]), s[16 + j], acc[16 + j]);
        }
      }
      if (!ok) {
#pragma unroll
        for (int j = 0; j < HALF; ++j) acc[j] = 0.f;
      }
      if (g.nsegs > 1) {
        // two partial slots per CTA: 1 for the segment that opens its tile,
        // 0 for a continuation
        float *wsl = a.ws + ((size_t)c * 2 + (g.seg == 0 ? 1 : 0)) * ((size_t)TN * BM);
#pragma unroll
        for (int j = 0; j < HALF; ++j) __stcg(wsl + (hf * HALF + j) * BM + row, acc[j]);
        __threadfence();
        named_bar(1, kEpiThreads);
        if (et == 0) *last_flag = atomicAdd(&a.tile_counters[g.tile], 1u) == (uint32_t)(g.nsegs - 1) ? 1 : 0;
        named_bar(1, kEpiThreads);
        const bool last = *last_flag;
        if (!last) continue;  // uniform across the epilogue threads
        __threadfence();
        const int c0 = c - g.seg;
#pragma unroll
        for (int j = 0; j < HALF; ++j) acc[j] = 0.f;
        for (int sg = 0; sg < g.nsegs; ++sg) {  // fixed order: deterministic sums
          const float *sl = a.ws + ((size_t)(c0 + sg) * 2 + (sg == 0 ? 1 : 0)) * ((size_t)TN * BM);
#pragma unroll
          for (int j = 0; j < HALF; ++j) acc[j] += __ldcg(sl + (hf * HALF + j) * BM + row);
        }
        if (et == 0) a.tile_counters[g.tile] = 0u;
      }
      // outputs straight from the accumulators: thread (row, half) holds
      // output feature `row` of its 32 tokens
      const int valid = sch.rows[ex] - tt * TN;
      if (EPI == kExpSwiGLU) {
        // gate rows 0..63 pair with up rows 64..127 (held by quarters 2, 3)
        if (q >= 2) {
#pragma unroll
          for (int j = 0; j < HALF; ++j) up_sm[(row - 64) * UP_PITCH + hf * HALF + j] = acc[j];
        }
        named_bar(1, kEpiThreads);
        if (q < 2) {
          __nv_bfloat16 *dst = a.act + (size_t)r0 * (a.N / 2) + nt * 64 + row;
#pragma unroll
          for (int j = 0; j < HALF; ++j) {
            const int tok = hf * HALF + j;
            if (tok < valid) dst[(size_t)tok * (a.N / 2)] = __float2bfloat16(silu(acc[j]) * up_sm[row * UP_PITCH + tok]);
          }
        }
      } else {
        // combine: each weighted row goes back to its source over NVLink
#pragma unroll
        for (int j = 0; j < HALF; ++j) {
          const int tok = hf * HALF + j;
          if (tok >= valid) continue;
          const int4 m = *reinterpret_cast<const int4 *>(a.meta + (size_t)(r0 + tok) * 4);
          a.combine[m.x][((size_t)m.y * a.k_top + m.z) * a.N + nt * BM + row] =
              __float2bfloat16(acc[j] * __int_as_float(m.w));
        }
        __threadfence_system();
        named_bar(1, kEpiThreads);
        // one count per (row, n-tile): the source expects N / 128 per row
        if (et < TN && et < valid) {
          const int src = a.meta[(size_t)(r0 + et) * 4];
          atomicAdd_system(a.combine_cnt[src], 1u);
        }
      }
      named_bar(1, kEpiThreads);  // up_sm is rewritten by the next tile
    }
  }

  __syncwarp();  // reconverge the elected-lane roles before the CTA barrier
  ptx::tc_fence_before();
  __syncthreads();
  if (a.trace && threadIdx.x == 0) a.trace[c * 4 + 3] = ptx::globaltimer_ns();
  if (warp == 0) ptx::tmem_dealloc(tmem, NP * TN);
  if (EPI == kExpSwiGLU && threadIdx.x == 0) finish_gate_up(a);
}

// ---------------------------------------------------------------- combine + residual + RMSNorm
// Waits until `expected` counts arrived (bounded), then
//   h[t] += sum_k c[t][k];   y[t] = rmsnorm(h[t]) * w;   and clears the counter.
__global__ void __launch_bounds__(512) combine_norm_kernel(const __nv_bfloat16 *__restrict__ c, int K,
                                                            __nv_bfloat16 *__restrict__ h,
                                                            const __nv_bfloat16 *__restrict__ w,
                                                            __nv_bfloat16 *__restrict__ y, int H, float eps,
                                                            uint32_t *cnt, uint32_t *dropped_step,
                                                            uint32_t *arrivals, int *status) {
  __shared__ float red[16];
  const int t = blockIdx.x;
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  if (threadIdx.x == 0) {
    // every kept assignment comes back as H/128 counted column tiles
    const uint32_t expected = ((uint32_t)gridDim.x * K - __ldcg(dropped_step)) * (uint32_t)(H / 128);
    bool ok = ptx::ld_acquire_sys(cnt) >= expected;
    if (!ok) {
      const uint64_t t0 = ptx::globaltimer_ns();
      while (!ok && ptx::globaltimer_ns() - t0 < kWaitBudgetNs) ok = ptx::ld_acquire_sys(cnt) >= expected;
      if (!ok) report_status(status, kStatusPeerTimeout);
    }
  }
  __syncwarp();
  __syncthreads();
  float v[8];
  float ss = 0.f;
  const int col = threadIdx.x * 8;
  if (col < H) {
    const uint4 hv = *reinterpret_cast<const uint4 *>(h + (size_t)t * H + col);
    const __nv_bfloat16 *he = reinterpret_cast<const __nv_bfloat16 *>(&hv);
    float s[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] = 0.f;
    for (int k = 0; k < K; ++k) {
      const uint4 cv = __ldcv(reinterpret_cast<const uint4 *>(c + ((size_t)t * K + k) * H + col));
      const __nv_bfloat16 *ce = reinterpret_cast<const __nv_bfloat16 *>(&cv);
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j] += __bfloat162float(ce[j]);
    }
    uint4 ov;
    __nv_bfloat16 *oe = reinterpret_cast<__nv_bfloat16 *>(&ov);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      oe[j] = __float2bfloat16(__bfloat162float(he[j]) + __bfloat162float(__float2bfloat16(s[j])));
      v[j] = __bfloat162float(oe[j]);
      ss += v[j] * v[j];
    }
    *reinterpret_cast<uint4 *>(h + (size_t)t * H + col) = ov;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
  __syncwarp();
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)blockDim.x / 32; ++i) tot += red[i];
  const float inv = rsqrtf(tot / H + eps);
  if (col < H) {
    const uint4 wv = *reinterpret_cast<const uint4 *>(w + col);
    const __nv_bfloat16 *we = reinterpret_cast<const __nv_bfloat16 *>(&wv);
    uint4 ov;
    ov.x = pack_bf16x2(v[0] * inv * __bfloat162float(we[0]), v[1] * inv * __bfloat162float(we[1]));
    ov.y = pack_bf16x2(v[2] * inv * __bfloat162float(we[2]), v[3] * inv * __bfloat162float(we[3]));
    ov.z = pack_bf16x2(v[4] * inv * __bfloat162float(we[4]), v[5] * inv * __bfloat162float(we[5]));
    ov.w = pack_bf16x2(v[6] * inv * __bfloat162float(we[6]), v[7] * inv * __bfloat162float(we[7]));
    *reinterpret_cast<uint4 *>(y + (size_t)t * H + col) = ov;
  }
  // the last token's CTA clears the counter for the next layer
  __syncwarp();
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(arrivals, 1u) == gridDim.x - 1) {
      *cnt = 0u;
      *dropped_step = 0u;
      *arrivals = 0u;
    }
  }
}

// activation quantisation for the down GEMM: bf16 [R, I] -> e4m3 + scale per
// 128 columns, for the valid rows of each expert only (rows_valid is known on
// the device alone, so the grid is fixed and strides over the valid units).
__global__ void __launch_bounds__(256) quantize_kernel(const __nv_bfloat16 *__restrict__ in, int I,
                                                       uint8_t *__restrict__ out, float *__restrict__ scale,
                                                       const uint32_t *rows_valid, int rows_per_expert,
                                                       int E_local) {
  __shared__ int prefix[33];
  const size_t R = (size_t)E_local * rows_per_expert;
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int nb = I / QB;
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E_local; ++e) {
      prefix[e] = acc;
      acc += min((int)__ldcg(rows_valid + e), rows_per_expert) * nb;
    }
    prefix[E_local] = acc;
  }
  __syncwarp();
  __syncthreads();
  const int total = prefix[E_local];
  const int lane = threadIdx.x % 32;
  const int warps = gridDim.x * (blockDim.x / 32);
  constexpr int U = 4;  // 128-column blocks per warp step: loads first, then math
  for (int u0 = (blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * U; u0 < total; u0 += warps * U) {
    uint2 raw[U];
    size_t off[U];
#pragma unroll
    for (int i = 0; i < U; ++i) {
      const int u = u0 + i;
      off[i] = ~size_t(0);
      if (u < total) {
        int ex = 0;
        while (u >= prefix[ex + 1]) ++ex;
        const int local = u - prefix[ex];
        const int r = ex * rows_per_expert + local / nb, blk = local % nb;
        off[i] = (size_t)r * I + blk * QB;
        raw[i] = *reinterpret_cast<const uint2 *>(in + off[i] + lane * 4);
      }
    }
#pragma unroll
    for (int i = 0; i < U; ++i) {
      if (off[i] == ~size_t(0)) continue;
      const __nv_bfloat16 *v = reinterpret_cast<const __nv_bfloat16 *>(&raw[i]);
      float f[4], m = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        f[j] = __bfloat162float(v[j]);
        m = fmaxf(m, fabsf(f[j]));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float sc = m > 0.f ? m / 448.f : 1.f, inv = 1.f / sc;
      uint32_t packed = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_fp8_e4m3 q(f[j] * inv);
        packed |= (uint32_t)(*reinterpret_cast<const uint8_t *>(&q)) << (8 * j);
      }
      *reinterpret_cast<uint32_t *>(out + off[i] + lane * 4) = packed;
      if (lane == 0) scale[(off[i] % I) / QB * R + off[i] / I] = sc;
    }
  }
}

}  // namespace moe

extern "C" int sched_moe_router(const void *x, const void *wr, int T, int H, int E, int K, int32_t *ids,
                                float *wts, cudaStream_t st) {
  if (T <= 0) return 0;
  if (E > 32 || K > moe::kMaxTopK || H % 256 != 0) return -1;
  launch_pdl(moe::router_topk_kernel, T, 32 * E, 0, st, static_cast<const __nv_bfloat16 *>(x),
             static_cast<const __nv_bfloat16 *>(wr), T, H, E, K, ids, wts);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int sched_moe_dispatch(const moe::DispatchArgs *a, cudaStream_t st) {
  if (a->H % moe::QB != 0 || a->world > moe::kMaxWorld || a->T < 0) return -1;
  // T == 0 still launches one CTA: every rank must announce completion
  if (a->K > moe::kMaxTopK) return -1;
  launch_pdl(moe::dispatch_kernel, a->T > 0 ? a->T : 1, 128, 0, st, *a);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

// w: [E_local * N, K] e4m3 (row-major), x: [E_local * rows, K] e4m3.
extern "C" int sched_moe_expert_gemm(int epi, const void *w, const void *x, const moe::ExpertArgs *args,
                                     cudaStream_t st) {
  moe::ExpertArgs a = *args;
  if (a.N % moe::BM != 0 || a.K % moe::BK != 0 || a.rows_per_expert % moe::TN != 0) return -1;
  if (a.E_local < 1 || a.E_local > moe::kMaxExperts || a.ws == nullptr || a.tile_counters == nullptr) return -1;
  a.n_tiles = a.N / moe::BM;
  a.t_tiles = a.rows_per_expert / moe::TN;
  a.ex_ld = a.K / moe::QB;
  int grid = a.grid;
  if (grid <= 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&grid, cudaDevAttrMultiProcessorCount, dev);
  }
  try {
    CUtensorMap tw = tmap::make_2d(w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a.E_local * a.N, a.K, a.K,
                                   moe::BM, moe::BK, CU_TENSOR_MAP_SWIZZLE_128B);
    CUtensorMap tx = tmap::make_2d(x, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a.E_local * a.rows_per_expert,
                                   a.K, a.K, moe::TN, moe::BK, CU_TENSOR_MAP_SWIZZLE_128B);
    if (epi == moe::kExpSwiGLU) {
      static bool s0 = false;
      if (!s0) {
        cudaFuncSetAttribute(moe::expert_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, moe::SMEM);
        s0 = true;
      }
      launch_pdl(moe::expert_gemm_kernel<0>, grid, moe::kThreads, moe::SMEM, st, tw, tx, a);
    } else {
      static bool s1 = false;
      if (!s1) {
        cudaFuncSetAttribute(moe::expert_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, moe::SMEM);
        s1 = true;
      }
      launch_pdl(moe::expert_gemm_kernel<1>, grid, moe::kThreads, moe::SMEM, st, tw, tx, a);
    }
  } catch (const std::exception &) {
    return -3;
  }
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int sched_moe_quantize(const void *in, int R, int I, void *out, float *scale,
                                  const uint32_t *rows_valid, int rows_per_expert, cudaStream_t st) {
  if (R <= 0) return 0;
  if (I % moe::QB != 0) return -1;
  const int E_local = R / rows_per_expert;
  if (E_local > 32 || R % rows_per_expert != 0) return -1;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  launch_pdl(moe::quantize_kernel, 2 * sms, 256, 0, st, static_cast<const __nv_bfloat16 *>(in), I,
             static_cast<uint8_t *>(out), scale, rows_valid, rows_per_expert, E_local);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int sched_moe_combine_norm(const void *c, int K, void *h, const void *w, void *y, int T, int H,
                                      float eps, uint32_t *cnt, uint32_t *dropped_step, uint32_t *arrivals,
                                      int *status, cudaStream_t st) {
  if (T <= 0) return 0;
  if (H % 8 != 0 || H / 8 > 512) return -1;
  launch_pdl(moe::combine_norm_kernel, T, 512, 0, st, static_cast<const __nv_bfloat16 *>(c), K,
             static_cast<__nv_bfloat16 *>(h), static_cast<const __nv_bfloat16 *>(w),
             static_cast<__nv_bfloat16 *>(y), H, eps, cnt, dropped_step, arrivals, status);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}
