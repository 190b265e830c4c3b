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
// One warp per token: logits over E experts (bf16 router weight [E, H]),
// top-k by value, weights = softmax over the selected logits (Mixtral).
__global__ void router_topk_kernel(const __nv_bfloat16 *__restrict__ x, const __nv_bfloat16 *__restrict__ wr,
                                   int T, int H, int E, int K, int32_t *__restrict__ ids,
                                   float *__restrict__ wts) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (warp >= T) return;
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  float logit[32];
  const __nv_bfloat16 *row = x + (size_t)warp * H;
  for (int e = 0; e < E; ++e) {
    float s = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
      const uint4 a = *reinterpret_cast<const uint4 *>(row + c);
      const uint4 b = *reinterpret_cast<const uint4 *>(wr + (size_t)e * H + c);
      const __nv_bfloat16 *ae = reinterpret_cast<const __nv_bfloat16 *>(&a);
      const __nv_bfloat16 *be = reinterpret_cast<const __nv_bfloat16 *>(&b);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += __bfloat162float(ae[j]) * __bfloat162float(be[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    logit[e] = s;
  }
  if (lane == 0) {
    int sel[kMaxTopK];
    float val[kMaxTopK];
    unsigned used = 0;
    for (int k = 0; k < K; ++k) {
      int best = -1;
      for (int e = 0; e < E; ++e)
        if (!(used >> e & 1u) && (best < 0 || logit[e] > logit[best])) best = e;
      used |= 1u << best;
      sel[k] = best;
      val[k] = logit[best];
    }
    float m = val[0], den = 0.f;
    for (int k = 0; k < K; ++k) den += __expf(val[k] - m);
    for (int k = 0; k < K; ++k) {
      ids[warp * K + k] = sel[k];
      wts[warp * K + k] = __expf(val[k] - m) / den;
    }
  }
}

// ---------------------------------------------------------------- dispatch
// One CTA (128 threads) per (token, k).
__global__ void __launch_bounds__(128) dispatch_kernel(const DispatchArgs a) {
  const int t = blockIdx.x / a.K, k = blockIdx.x % a.K;
  __shared__ int slot_s;
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  if (t >= a.T) goto announce;  // a rank with no tokens still announces completion
  {
  const int e = a.ids[t * a.K + k];
  const int owner = e / a.E_local, le = e % a.E_local;
  if (threadIdx.x == 0) {
    const uint32_t s = atomicAdd_system(a.counter[owner] + le, 1u);
    slot_s = (int)s < a.capacity ? (int)s : -1;
    if (slot_s < 0) {
      atomicAdd(a.dropped_step, 1u);
      if (a.dropped_total) atomicAdd(a.dropped_total, 1u);
    }
  }
  __syncthreads();
  const int slot = slot_s;
  if (slot < 0) {
    // dropped by the capacity cap: its combine row contributes zero
    __nv_bfloat16 *c = a.combine_local + ((size_t)t * a.K + k) * a.H;
    for (int col = threadIdx.x * 8; col < a.H; col += 128 * 8)
      *reinterpret_cast<uint4 *>(c + col) = make_uint4(0, 0, 0, 0);
  } else {
    const size_t row = (size_t)le * a.rows_per_expert + slot;
    const __nv_bfloat16 *src = a.x + (size_t)t * a.H;
    uint8_t *dst = a.slab[owner] + row * a.H;
    float *dscale = a.slab_scale[owner] + row * (a.H / QB);
    // each warp quantises 128-column blocks: amax -> scale -> e4m3
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
      *reinterpret_cast<uint32_t *>(dst + blk * QB + lane * 4) = packed;
      if (lane == 0) dscale[blk] = scale;
    }
    if (threadIdx.x == 0) {
      int4 meta = make_int4(a.rank, t, k, __float_as_int(a.wts[t * a.K + k]));
      *reinterpret_cast<int4 *>(a.slab_meta[owner] + row * 4) = meta;
    }
  }
  }
announce:
  // the last dispatch CTA of this rank announces completion to every owner
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t fin = atomicAdd(a.local_done, 1u);
    if (fin == gridDim.x - 1) {
      *a.local_done = 0u;
      __threadfence_system();
      for (int r = 0; r < a.world; ++r) atomicAdd_system(a.done[r], 1u);
    }
  }
}

// ---------------------------------------------------------------- fp8 expert GEMM
constexpr int BM = 128;
constexpr int BK = 128;  // fp8 elements per stage = 128 bytes
constexpr int TN = 64;   // rows (tokens) per tile
constexpr int kThreads = 192;
constexpr int W_BYTES = BM * BK;
constexpr int X_BYTES = TN * BK;
constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
constexpr int STAGES = 8;
constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 512;

// gate/up: the last CTA publishes the row counts for the down GEMM and
// clears the receive counters (every CTA has read its rows by now).
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
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + STAGES * STAGE_BYTES);
  uint64_t *full = bars, *empty = bars + STAGES, *p_full = bars + 2 * STAGES, *p_empty = bars + 2 * STAGES + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 4);
  int *valid_s = reinterpret_cast<int *>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // n-tiles fastest, token tiles next: the (usually few) valid token tiles
  // occupy the first CTAs; the rest exit right after the row-count check
  int tile = blockIdx.x;
  const int nt = tile % a.n_tiles;
  tile /= a.n_tiles;
  const int tt = tile % a.t_tiles;
  const int ex = tile / a.t_tiles;
  const int kb_total = a.K / BK;

  ptx::pdl_launch_dependents();
  // rows of this expert: gate/up waits for every source's dispatch first
  if (threadIdx.x == 0) {
    ptx::pdl_wait();
    int rows;
    if (EPI == kExpSwiGLU) {
      bool ok = ptx::ld_acquire_sys(a.done) >= (uint32_t)a.world;
      if (!ok) {
        const uint64_t t0 = ptx::globaltimer_ns();
        while (!ok && ptx::globaltimer_ns() - t0 < kWaitBudgetNs) ok = ptx::ld_acquire_sys(a.done) >= (uint32_t)a.world;
        if (!ok) report_status(a.status, kStatusPeerTimeout);
      }
      rows = min((int)ptx::ld_acquire_sys(a.counter + ex), a.capacity);
    } else {
      rows = (int)__ldcg(a.rows_valid + ex);
    }
    *valid_s = rows;
  }
  __syncthreads();
  const int valid = *valid_s;
  const bool active = tt * TN < valid;
  if (!active) {
    if (EPI == kExpSwiGLU && threadIdx.x == 0) finish_gate_up(a);
    return;
  }
  if (warp == 0) {
    ptx::tmem_alloc(tmem_slot, 2 * TN);
    ptx::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&p_full[i], 1);
      ptx::mbar_init(&p_empty[i], 128);
    }
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

  if (active && warp == 0) {
    if (ptx::elect_one()) {
      // the slab rows arrived through peers' generic stores; TMA reads them
      ptx::fence_proxy_async_global();
      for (int kb = 0; kb < kb_total; ++kb) {
        const int s = kb % STAGES;
        if (!ptx::mbar_wait(&empty[s], ((kb / STAGES) & 1) ^ 1)) {
          report_status(a.status, kStatusMmaTimeout);
          break;
        }
        uint8_t *st = base + s * STAGE_BYTES;
        ptx::mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
        ptx::tma_load_2d(st, &tmW, &full[s], kb * BK, ex * a.N + nt * BM);
        ptx::tma_load_2d(st + W_BYTES, &tmX, &full[s], kb * BK, ex * a.rows_per_expert + tt * TN);
      }
    }
  } else if (active && warp == 1) {
    if (ptx::elect_one()) {
      constexpr uint32_t idesc = ptx::idesc_e4m3(BM, TN);
      for (int kb = 0; kb < kb_total; ++kb) {
        const int s = kb % STAGES, pb = kb & 1;
        if (!ptx::mbar_wait(&full[s], (kb / STAGES) & 1) ||
            !ptx::mbar_wait(&p_empty[pb], ((kb >> 1) & 1) ^ 1)) {
          report_status(a.status, kStatusTmaTimeout);
          break;
        }
        ptx::tc_fence_after();
        uint8_t *st = base + s * STAGE_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 32; ++kk) {
          const uint64_t da = ptx::smem_desc(st + kk * 32, 16, 1024, ptx::kLayoutSW128);
          const uint64_t db = ptx::smem_desc(st + W_BYTES + kk * 32, 16, 1024, ptx::kLayoutSW128);
          ptx::mma_f8_ss(tmem + pb * TN, da, db, idesc, kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit(&empty[s]);
        ptx::mma_commit(&p_full[pb]);
      }
    }
  } else if (active && warp >= 2) {
    // promotion: acc[t] += partial[row][t] * s_w[kb] * s_x[t][kb]
    const int q = warp & 3, row = q * 32 + lane;
    float acc[TN];
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[j] = 0.f;
    const float *sw = a.w_scale + ((size_t)ex * a.n_tiles + nt) * kb_total;
    const int r0 = ex * a.rows_per_expert + tt * TN;
    bool ok = true;
    for (int kb = 0; kb < kb_total && ok; ++kb) {
      const int pb = kb & 1;
      if (!ptx::mbar_wait(&p_full[pb], (kb >> 1) & 1)) {
        report_status(a.status, kStatusEpilogueTimeout);
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      const float swk = __ldg(sw + kb);
#pragma unroll
      for (int c = 0; c < TN / 16; ++c) {
        uint32_t r[16];
        ptx::tmem_ld16(tmem + pb * TN + ((uint32_t)(q * 32) << 16) + c * 16, r);
        ptx::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j)
          acc[c * 16 + j] += __uint_as_float(r[j]) * swk * __ldg(a.x_scale + (size_t)(r0 + c * 16 + j) * a.ex_ld + kb);
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(&p_empty[pb]);
    }
    // stage the tile through shared memory (reusing the ring) for row-wise writes
    __syncwarp();
    float *tile_sm = reinterpret_cast<float *>(base);  // [TN][BM + 4]
    named_bar(1, 128);  // the ring is idle: every MMA has been consumed
#pragma unroll
    for (int j = 0; j < TN; ++j) tile_sm[j * (BM + 4) + row] = acc[j];
    named_bar(1, 128);
    const int et = threadIdx.x - 64;
    if (EPI == kExpSwiGLU) {
      // 64 gate rows + their 64 up rows -> 64 act columns per token
      for (int idx = et; idx < TN * 8; idx += 128) {
        const int tj = idx / 8, c = (idx % 8) * 8;
        if (tt * TN + tj >= valid) continue;
        const float *v = tile_sm + tj * (BM + 4);
        uint4 o;
        o.x = pack_bf16x2(silu(v[c]) * v[c + 64], silu(v[c + 1]) * v[c + 65]);
        o.y = pack_bf16x2(silu(v[c + 2]) * v[c + 66], silu(v[c + 3]) * v[c + 67]);
        o.z = pack_bf16x2(silu(v[c + 4]) * v[c + 68], silu(v[c + 5]) * v[c + 69]);
        o.w = pack_bf16x2(silu(v[c + 6]) * v[c + 70], silu(v[c + 7]) * v[c + 71]);
        *reinterpret_cast<uint4 *>(a.act + (size_t)(r0 + tj) * (a.N / 2) + nt * 64 + c) = o;
      }
    } else {
      // combine: row (weighted) back to its source over NVLink
      for (int idx = et; idx < TN * 16; idx += 128) {
        const int tj = idx / 16, c = (idx % 16) * 8;
        if (tt * TN + tj >= valid) continue;
        const int4 m = *reinterpret_cast<const int4 *>(a.meta + (size_t)(r0 + tj) * 4);
        const float w = __int_as_float(m.w);
        const float *v = tile_sm + tj * (BM + 4);
        uint4 o;
        o.x = pack_bf16x2(v[c] * w, v[c + 1] * w);
        o.y = pack_bf16x2(v[c + 2] * w, v[c + 3] * w);
        o.z = pack_bf16x2(v[c + 4] * w, v[c + 5] * w);
        o.w = pack_bf16x2(v[c + 6] * w, v[c + 7] * w);
        __nv_bfloat16 *dst = a.combine[m.x] + ((size_t)m.y * a.k_top + m.z) * a.N + nt * BM + c;
        *reinterpret_cast<uint4 *>(dst) = o;
      }
      __threadfence_system();
      named_bar(1, 128);
      // one count per (row, n-tile) pushed: the source expects N/128 per row
      for (int tj = et; tj < TN; tj += 128) {
        if (tt * TN + tj >= valid) continue;
        const int src = a.meta[(size_t)(r0 + tj) * 4];
        atomicAdd_system(a.combine_cnt[src], 1u);
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) ptx::tmem_dealloc(tmem, 2 * TN);
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

// activation quantisation for the down GEMM: bf16 [R, I] -> e4m3 + scale per 128
__global__ void quantize_kernel(const __nv_bfloat16 *__restrict__ in, int I, uint8_t *__restrict__ out,
                                float *__restrict__ scale, const uint32_t *rows_valid, int rows_per_expert) {
  const int r = blockIdx.x, blk = blockIdx.y;  // one warp per (row, 128-block)
  const int lane = threadIdx.x;
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int ex = r / rows_per_expert;
  if (r % rows_per_expert >= (int)__ldcg(rows_valid + ex)) return;
  const uint2 u = *reinterpret_cast<const uint2 *>(in + (size_t)r * I + blk * QB + lane * 4);
  const __nv_bfloat16 *v = reinterpret_cast<const __nv_bfloat16 *>(&u);
  float f[4], m = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[j] = __bfloat162float(v[j]);
    m = fmaxf(m, fabsf(f[j]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float s = m > 0.f ? m / 448.f : 1.f, inv = 1.f / s;
  uint32_t packed = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_fp8_e4m3 q(f[j] * inv);
    packed |= (uint32_t)(*reinterpret_cast<const uint8_t *>(&q)) << (8 * j);
  }
  *reinterpret_cast<uint32_t *>(out + (size_t)r * I + blk * QB + lane * 4) = packed;
  if (lane == 0) scale[(size_t)r * (I / QB) + blk] = s;
}

}  // namespace moe

extern "C" int sched_moe_router(const void *x, const void *wr, int T, int H, int E, int K, int32_t *ids,
                                float *wts, cudaStream_t st) {
  if (T <= 0) return 0;
  if (E > 32 || K > moe::kMaxTopK || H % 256 != 0) return -1;
  launch_pdl(moe::router_topk_kernel, (T + 3) / 4, 128, 0, st, static_cast<const __nv_bfloat16 *>(x),
             static_cast<const __nv_bfloat16 *>(wr), T, H, E, K, ids, wts);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int sched_moe_dispatch(const moe::DispatchArgs *a, cudaStream_t st) {
  if (a->H % moe::QB != 0 || a->world > moe::kMaxWorld || a->T < 0) return -1;
  // T == 0 still launches one CTA: every rank must announce completion
  launch_pdl(moe::dispatch_kernel, a->T > 0 ? a->T * a->K : 1, 128, 0, st, *a);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

// w: [E_local * N, K] e4m3 (row-major), x: [E_local * rows, K] e4m3.
extern "C" int sched_moe_expert_gemm(int epi, const void *w, const void *x, const moe::ExpertArgs *args,
                                     cudaStream_t st) {
  moe::ExpertArgs a = *args;
  if (a.N % moe::BM != 0 || a.K % moe::BK != 0 || a.rows_per_expert % moe::TN != 0) return -1;
  a.n_tiles = a.N / moe::BM;
  a.t_tiles = a.rows_per_expert / moe::TN;
  a.ex_ld = a.K / moe::QB;
  try {
    CUtensorMap tw = tmap::make_2d(w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a.E_local * a.N, a.K, a.K,
                                   moe::BM, moe::BK, CU_TENSOR_MAP_SWIZZLE_128B);
    CUtensorMap tx = tmap::make_2d(x, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a.E_local * a.rows_per_expert,
                                   a.K, a.K, moe::TN, moe::BK, CU_TENSOR_MAP_SWIZZLE_128B);
    const int grid = a.E_local * a.n_tiles * a.t_tiles;
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
  launch_pdl(moe::quantize_kernel, dim3(R, I / moe::QB), 32, 0, st, static_cast<const __nv_bfloat16 *>(in), I,
             static_cast<uint8_t *>(out), scale, rows_valid, rows_per_expert);
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
