// attention_prefill.cu -- causal attention of prefill chunks over the paged KV
// cache on the sm_100a tensor cores (tcgen05, accumulators in TMEM, KV pages
// fed by TMA).
//
// Problem: a query tile is up to 128 consecutive query rows of one request
// (row i at absolute position q_pos0 + i) and one query head; row i attends
// to the request's KV tokens [0, q_pos0 + i]. This covers a whole prompt and
// a chunk appended to a cached prefix alike. The cache layout is
// [pages, Hkv, 16, 128] bf16: one 4-D TMA box fetches one page of one KV
// head (4 KB, 128-byte swizzle).
//
// Tensor-core mapping (one CTA per (tile, head)):
//   S[128 q x 128 tok] = Q[128 q x 128 d] . K_blk^T    kind::f16, Q and K from smem (K-major)
//   O[128 q x 128 d]  += P[128 q x 128 tok] . V_blk    P from TMEM, V from smem (MN-major)
// S, P and O live in TMEM with one query row per lane, so each of the 128
// softmax threads owns one row: its max, exponentials and sum need no
// shuffles or shared-memory reductions, and P goes back to the tensor core
// through TMEM (tcgen05.st, bf16 pairs) without a trip through shared memory.
// TMEM columns: S double-buffered at [0,128) and [128,256), O at [256,384),
// P double-buffered at [384,448) and [448,512); so the MMA warp computes S of
// block b+1 while the softmax warps turn S of block b into P.
//
// Online softmax with a lazy rescale: a row keeps the running maximum m it
// used for its exponentials until a block raises the maximum by more than
// 2^8 (8 in log2 units). Until then P <= 2^8 (exact enough in bf16, and the
// fp32 O and l accumulate it without overflow); O/l is the same for any m, so
// the result is exact softmax. Only a rescale touches O in TMEM (load,
// scale, store), after the previous block's PV product has completed. For
// the causal diagonal and for random data this happens in the first block
// and almost never after.
//
// Warp roles (192 threads): warps 0-3 Q staging, softmax and output (TMEM lane
// quarter = warp), warp 4 TMA producer, warp 5 MMA issuer. KV blocks of 128
// tokens flow through a three-stage ring of 64 KB (K and V with separate
// barriers, so S can start before V has landed).
//
// Reference: the woven FlashInfer prefill kernel (jc-su/sched-pass
// test/py/test_flashinfer_prefill.py:1-146) is the hot path this replaces;
// the tile order (pi over prefill tiles, longest first) is set by the host
// (engine.order_prefill_tiles, after ROADMAP.md:450-451).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>

#include "common.cuh"
#include "sched/ptx.cuh"
#include "tmap.h"

namespace pf {

constexpr int D = 128;
constexpr int PS = 16;                  // tokens per page
constexpr int BQ = 128;                 // query rows per tile (MMA M)
constexpr int BKV = 128;                // KV tokens per block
constexpr int PAGES_PER_BLK = BKV / PS;
constexpr int STAGES = 3;
constexpr int kThreads = 192;
constexpr int kSoftmaxThreads = 128;
constexpr int HALF = 128 * 128;         // bytes of a 64-column half of a 128-row bf16 tile
constexpr int TILE_BYTES = 2 * HALF;    // 128 rows x 128 bf16
// A K or V block is 8 page-head boxes of 4 KB (tmap::make_kv_pages):
// [row group][column half][8 rows][128 bytes]; 8-row atoms of one column
// half are 2 KB apart and the other half's atom is at +1 KB. (Q keeps the
// plain layout: each half is a 16 KB plane with atoms 1 KB apart.)
constexpr int PAGE_BYTES = PS * 256;
constexpr int ATOM = 1024;
constexpr int ATOM_PAIR = 2048;
constexpr int STAGE_BYTES = 2 * TILE_BYTES;  // K + V
constexpr int TMEM_COLS = 512;          // S0 [0,128), S1 [128,256), O [256,384), P0/P1 [384,512)
constexpr int O_COL = 256;
constexpr int P_COL = 384;              // 64 columns (128 bf16) per P buffer
constexpr float kRescaleLog2 = 8.f;     // lazy-rescale threshold (log2 units)

struct QTile {
  int32_t req;     // request index (row of block table / kv_lens)
  int32_t q_row0;  // first row of this tile in the packed q / out tensors
  int32_t nq;      // rows in this tile (<= 128; 0 = empty tile)
  int32_t q_pos0;  // absolute position of the first row
};

struct Params {
  const __nv_bfloat16 *q;  // [T, Hq, D]
  __nv_bfloat16 *out;      // [T, Hq, D]
  const int32_t *block_table;
  int bt_stride;
  const int32_t *kv_lens;
  const QTile *tiles;
  int Hq, Hkv;
  float scale_log2;  // softmax scale * log2(e)
  int num_pages;     // pages of the cache: ids outside [0, num_pages) are reported and read as zeros
  int total_rows;    // rows of the cache tensor maps (pages * Hkv * 16): an out-of-range box row
  int *status;
};

struct Shared {
  uint64_t k_full[STAGES], v_full[STAGES], kv_empty[STAGES];
  uint64_t s_ready[2], s_free[2], p_ready[2], pv_done[2];
  uint64_t q_full;
  uint32_t tmem_base;
};

constexpr int SMEM = 1024 + TILE_BYTES /*Q*/ + STAGES * STAGE_BYTES + (int)sizeof(Shared);
static_assert(SMEM <= 232448, "shared memory per CTA");

__device__ __forceinline__ uint32_t swz(uint32_t row, uint32_t byte_in_row) {
  // 128-byte swizzle: the 16-byte chunk index is XORed with (row % 8).
  return row * 128u + ((((byte_in_row >> 4) ^ (row & 7u)) << 4) | (byte_in_row & 15u));
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const Params p) {
  const int task = blockIdx.x;
  const QTile tile = p.tiles[task / p.Hq];
  const int hq = task % p.Hq;
  const int kvh = hq / (p.Hq / p.Hkv);
  if (tile.nq <= 0) return;  // empty (padding) tile: uniform across the CTA

  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *q_sm = base;
  uint8_t *stages = q_sm + TILE_BYTES;
  Shared &sh = *reinterpret_cast<Shared *>(stages + STAGES * STAGE_BYTES);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  // ------------------------------------------------------------------ setup
  if (warp == 0) {
    ptx::tmem_alloc(&sh.tmem_base, TMEM_COLS);
    ptx::tmem_relinquish();
  }
  if (threadIdx.x == 32 * 4) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&sh.k_full[s], 1);
      ptx::mbar_init(&sh.v_full[s], 1);
      ptx::mbar_init(&sh.kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&sh.s_ready[i], 1);
      ptx::mbar_init(&sh.s_free[i], kSoftmaxThreads);
      ptx::mbar_init(&sh.p_ready[i], kSoftmaxThreads);
      ptx::mbar_init(&sh.pv_done[i], 1);
    }
    ptx::mbar_init(&sh.q_full, 1);
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tmQ);
    ptx::prefetch_tmap(&tmK);
    ptx::prefetch_tmap(&tmV);
  }
  ptx::pdl_launch_dependents();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  ptx::pdl_wait();  // q and the cache are written by the kernels before this one

  const int kv_len = p.kv_lens[tile.req];
  const int kv_stop = min(kv_len, tile.q_pos0 + tile.nq);  // the last row sees [0, kv_stop)
  const int nblk = kv_stop > 0 ? (kv_stop + BKV - 1) / BKV : 0;

  if (warp == 4) {
    // ============================================================ producer
    if (lane == 0 && nblk > 0) {
      const int32_t *bt = p.block_table + (size_t)tile.req * p.bt_stride;
      const int last_page = (kv_stop + PS - 1) / PS;
      // a block's page ids are loaded together and one block ahead of its
      // TMA issue, so their latency hides behind the wait for a free stage
      int ids_next[PAGES_PER_BLK];
      auto load_ids = [&](int b, int *ids) {
        const int pg0 = b * PAGES_PER_BLK;
#pragma unroll
        for (int pi = 0; pi < PAGES_PER_BLK; ++pi)
          ids[pi] = pg0 + pi < last_page ? __ldg(bt + pg0 + pi) : -1;
      };
      load_ids(0, ids_next);
      // Q: 128 rows of this head from q_row0 (rows past nq are other tiles'
      // rows or out-of-range zeros; they only feed rows that are never stored)
      ptx::mbar_arrive_expect_tx(&sh.q_full, TILE_BYTES);
      ptx::tma_load_3d(q_sm, &tmQ, &sh.q_full, 0, hq, tile.q_row0);
      ptx::tma_load_3d(q_sm + HALF, &tmQ, &sh.q_full, 64, hq, tile.q_row0);
      for (int b = 0; b < nblk; ++b) {
        int ids[PAGES_PER_BLK];
#pragma unroll
        for (int pi = 0; pi < PAGES_PER_BLK; ++pi) ids[pi] = ids_next[pi];
        if (b + 1 < nblk) load_ids(b + 1, ids_next);
        const int s = b % STAGES;
        if (!ptx::mbar_wait(&sh.kv_empty[s], ((b / STAGES) & 1) ^ 1, kWaitBudgetNs)) {
          report_status(p.status, kStatusMmaTimeout);
          break;
        }
        uint8_t *kst = stages + s * STAGE_BYTES;
        uint8_t *vst = kst + TILE_BYTES;
        ptx::mbar_arrive_expect_tx(&sh.k_full[s], TILE_BYTES);
        ptx::mbar_arrive_expect_tx(&sh.v_full[s], TILE_BYTES);
#pragma unroll
        for (int pi = 0; pi < PAGES_PER_BLK; ++pi) {
          int page = ids[pi];
          if (b * PAGES_PER_BLK + pi < last_page && (page < 0 || page >= p.num_pages)) {
            report_bad_index(p.status, kSitePrefillPage, page);  // read as a zero box
            page = -1;
          }
          // pages past the last one (and bad ids): an out-of-range box reads zeros
          const int rg = page < 0 ? p.total_rows / 8 : (page * p.Hkv + kvh) * (PS / 8);
          ptx::tma_load_4d(kst + pi * PAGE_BYTES, &tmK, &sh.k_full[s], 0, 0, 0, rg);
        }
#pragma unroll
        for (int pi = 0; pi < PAGES_PER_BLK; ++pi) {
          int page = ids[pi];
          if (page >= p.num_pages) page = -1;
          const int rg = page < 0 ? p.total_rows / 8 : (page * p.Hkv + kvh) * (PS / 8);
          ptx::tma_load_4d(vst + pi * PAGE_BYTES, &tmV, &sh.v_full[s], 0, 0, 0, rg);
        }
      }
    }
  } else if (warp == 5) {
    // ============================================================ MMA issuer
    if (lane == 0 && nblk > 0) {
      constexpr uint32_t idS = ptx::idesc_f16(BQ, BKV, 1, false, false);  // Q, K both K-major
      constexpr uint32_t idO = ptx::idesc_f16(BQ, D, 1, false, true);     // P (TMEM), V MN-major
      bool ok = ptx::mbar_wait(&sh.q_full, 0, kWaitBudgetNs);
      auto issue_s = [&](int b) -> bool {
        const int s = b % STAGES, sb = b & 1;
        if (!ptx::mbar_wait(&sh.k_full[s], (b / STAGES) & 1, kWaitBudgetNs)) return false;
        if (!ptx::mbar_wait(&sh.s_free[sb], ((b >> 1) & 1) ^ 1, kWaitBudgetNs)) return false;
        ptx::tc_fence_after();
        const uint8_t *kst = stages + s * STAGE_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qoff = (kk / 4) * HALF + (kk % 4) * 32;
          const uint32_t koff = (kk / 4) * ATOM + (kk % 4) * 32;
          ptx::mma_f16_ss(tmem + sb * BKV, ptx::smem_desc(q_sm + qoff, 16, 1024, ptx::kLayoutSW128),
                          ptx::smem_desc(kst + koff, 16, ATOM_PAIR, ptx::kLayoutSW128), idS, kk > 0);
        }
        ptx::mma_commit(&sh.s_ready[sb]);
        return true;
      };
      auto issue_o = [&](int b) -> bool {
        const int s = b % STAGES, pb = b & 1;
        if (!ptx::mbar_wait(&sh.v_full[s], (b / STAGES) & 1, kWaitBudgetNs)) return false;
        if (!ptx::mbar_wait(&sh.p_ready[pb], (b >> 1) & 1, kWaitBudgetNs)) return false;
        ptx::tc_fence_after();
        const uint8_t *vst = stages + s * STAGE_BYTES + TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          // A = P in TMEM: 16 tokens per MMA = 8 columns of bf16 pairs;
          // B = V, MN-major: 64 d per 128-byte row, other d half at +1 KB (LBO),
          // 8-token groups at +2 KB (SBO); 16 tokens per MMA = +4 KB.
          const uint8_t *bv = vst + kk * 2 * ATOM_PAIR;
          ptx::mma_f16_ts(tmem + O_COL, tmem + P_COL + pb * (BKV / 2) + kk * 8,
                          ptx::smem_desc(bv, ATOM, ATOM_PAIR, ptx::kLayoutSW128), idO,
                          (b > 0 || kk > 0) ? 1u : 0u);
        }
        ptx::mma_commit(&sh.pv_done[pb]);
        ptx::mma_commit(&sh.kv_empty[s]);  // S(b) and PV(b) have read stage s
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int b = 0; ok && b < nblk; ++b) {
        if (b + 1 < nblk && !issue_s(b + 1)) { ok = false; break; }
        if (!issue_o(b)) { ok = false; break; }
      }
      if (!ok) report_status(p.status, kStatusTmaTimeout);
    }
  } else {
    // ============================================================ softmax + output
    const int t = threadIdx.x;  // query row of the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    // this row sees tokens [0, qlim]
    const int qlim = min(tile.q_pos0 + t, kv_stop - 1);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int b = 0; b < nblk; ++b) {
      const int sb = b & 1;
      if (!ptx::mbar_wait(&sh.s_ready[sb], (b >> 1) & 1, kWaitBudgetNs)) {
        report_status(p.status, kStatusMmaTimeout);
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      uint32_t s[8][16];
#pragma unroll
      for (int i = 0; i < 8; ++i) ptx::tmem_ld16(tmem + lane_off + sb * BKV + i * 16, s[i]);
      ptx::tmem_ld_wait();
      ptx::tc_fence_before();
      ptx::mbar_arrive(&sh.s_free[sb]);
      // causal / length mask (only the blocks that reach past qlim); the row
      // max is 4 independent chains of three-input maxima
      const int tok0 = b * BKV;
      if (tok0 + BKV - 1 > qlim) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int k = 0; k < 16; ++k)
            if (tok0 + i * 16 + k > qlim) s[i][k] = __float_as_uint(-INFINITY);
      }
      float mxp[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int k = 0; k < 16; k += 2)
          mxp[(i * 8 + k / 2) & 3] =
              fmax3(mxp[(i * 8 + k / 2) & 3], __uint_as_float(s[i][k]), __uint_as_float(s[i][k + 1]));
      const float mx = fmax3(mxp[0], mxp[1], fmaxf(mxp[2], mxp[3]));
      const float m_cand = fmaxf(m_run, mx * p.scale_log2);
      // lazy rescale. A row moves its reference max only when its own max
      // grew past the threshold, so its arithmetic never depends on the other
      // rows of its warp (or on how a prompt was cut into tiles and chunks);
      // the TMEM accesses are warp-collective, so the warp runs them when any
      // of its rows rescales, and the other rows scale by 1.
      const bool grow = m_cand > m_run + kRescaleLog2;
      if (__any_sync(0xffffffffu, grow)) {
        float f = 1.f;
        if (grow) {
          f = m_run == -INFINITY ? 0.f : ex2_approx(m_run - m_cand);
          m_run = m_cand;
        }
        l_run *= f;
        if (b > 0) {  // O holds blocks [0, b): wait for PV(b-1), then scale it in place
          const int pb = (b - 1) & 1;
          const bool got = ptx::mbar_wait(&sh.pv_done[pb], ((b - 1) >> 1) & 1, kWaitBudgetNs);
          if (!__all_sync(0xffffffffu, got)) {
            report_status(p.status, kStatusMmaTimeout);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            uint32_t o[16];
            ptx::tmem_ld16(tmem + lane_off + O_COL + i * 16, o);
            ptx::tmem_ld_wait();
#pragma unroll
            for (int k = 0; k < 16; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * f);
            ptx::tmem_st16(tmem + lane_off + O_COL + i * 16, o);
          }
          ptx::tmem_st_wait();
        }
      }
      // P = 2^(s * scale - m), row sum; an all-masked row so far has m = -inf
      // and only -inf scores, which give 0 with an offset of 0
      const float neg = m_run == -INFINITY ? 0.f : -m_run;
      const uint64_t sc2 = f32x2_splat(p.scale_log2), ng2 = f32x2_splat(neg);
      uint32_t pk[4][16];  // P row as bf16 pairs: token 2c in the low half of column c
      float rsp[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float x0, x1;
          ffma2(x0, x1, __uint_as_float(s[i][2 * k]), __uint_as_float(s[i][2 * k + 1]), sc2, ng2);
          const float a = ex2_approx(x0), c = ex2_approx(x1);
          fadd2(rsp[k & 3][0], rsp[k & 3][1], a, c);
          pk[i / 2][(i % 2) * 8 + k] = pack_bf16x2(a, c);
        }
      }
      l_run += ((rsp[0][0] + rsp[0][1]) + (rsp[1][0] + rsp[1][1])) +
               ((rsp[2][0] + rsp[2][1]) + (rsp[3][0] + rsp[3][1]));
      // P buffer b&1 was last read by PV(b-2)
      const bool pfree = b < 2 || ptx::mbar_wait(&sh.pv_done[sb], ((b - 2) >> 1) & 1, kWaitBudgetNs);
      if (!__all_sync(0xffffffffu, pfree)) {
        report_status(p.status, kStatusMmaTimeout);
        ok = false;
        break;
      }
      ptx::tc_fence_after();
#pragma unroll
      for (int i = 0; i < 4; ++i) ptx::tmem_st16(tmem + lane_off + P_COL + sb * (BKV / 2) + i * 16, pk[i]);
      ptx::tmem_st_wait();
      ptx::tc_fence_before();
      ptx::mbar_arrive(&sh.p_ready[sb]);
    }
    // output: O / l for this row
    if (ok && nblk > 0) {
      const int pb = (nblk - 1) & 1;
      const bool got = ptx::mbar_wait(&sh.pv_done[pb], ((nblk - 1) >> 1) & 1, kWaitBudgetNs);
      if (__all_sync(0xffffffffu, got)) {
        ptx::tc_fence_after();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        uint4 *dst = reinterpret_cast<uint4 *>(p.out + ((size_t)(tile.q_row0 + t) * p.Hq + hq) * D);
        uint32_t o[8][16];
#pragma unroll
        for (int i = 0; i < 8; ++i) ptx::tmem_ld16(tmem + lane_off + O_COL + i * 16, o[i]);
        ptx::tmem_ld_wait();
        if (t < tile.nq) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int h = 0; h < 2; ++h)
              dst[i * 2 + h] = make_uint4(
                  pack_bf16x2(__uint_as_float(o[i][8 * h + 0]) * inv, __uint_as_float(o[i][8 * h + 1]) * inv),
                  pack_bf16x2(__uint_as_float(o[i][8 * h + 2]) * inv, __uint_as_float(o[i][8 * h + 3]) * inv),
                  pack_bf16x2(__uint_as_float(o[i][8 * h + 4]) * inv, __uint_as_float(o[i][8 * h + 5]) * inv),
                  pack_bf16x2(__uint_as_float(o[i][8 * h + 6]) * inv, __uint_as_float(o[i][8 * h + 7]) * inv));
        }
      } else {
        report_status(p.status, kStatusMmaTimeout);
      }
    }
  }

  __syncwarp();  // reconverge single-lane roles before the CTA barrier
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) ptx::tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace pf

extern "C" int sched_attn_prefill_tile_rows() { return pf::BQ; }

// q, out [q_rows, Hq, 128] bf16; k_cache/v_cache [num_pages, Hkv, 16, 128] bf16;
// tiles [num_tiles] (req, q_row0, nq <= 128, q_pos0), launched in the given
// order (tile-major, heads minor). Returns 0 on success.
extern "C" int sched_attn_prefill(const void *q, int q_rows, void *out, const void *k_cache,
                                  const void *v_cache, int num_pages, const int32_t *block_table,
                                  int bt_stride, const int32_t *kv_lens, const void *tiles,
                                  int num_tiles, int Hq, int Hkv, int page_size, float sm_scale,
                                  int *status, cudaStream_t st) {
  if (num_tiles <= 0) return 0;
  if (page_size != pf::PS || Hkv <= 0 || Hq % Hkv != 0 || num_pages <= 0 || q_rows <= 0) return -1;
  pf::Params p;
  p.q = static_cast<const __nv_bfloat16 *>(q);
  p.out = static_cast<__nv_bfloat16 *>(out);
  p.block_table = block_table;
  p.bt_stride = bt_stride;
  p.kv_lens = kv_lens;
  p.tiles = static_cast<const pf::QTile *>(tiles);
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.num_pages = num_pages;
  p.total_rows = num_pages * Hkv * pf::PS;
  p.status = status;
  try {
    const uint64_t rows = (uint64_t)num_pages * Hkv * pf::PS;
    CUtensorMap tq = tmap::make_3d(q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                                   {(uint64_t)pf::D, (uint64_t)Hq, (uint64_t)q_rows},
                                   {(uint64_t)pf::D * 2, (uint64_t)Hq * pf::D * 2}, {64u, 1u, 128u},
                                   CU_TENSOR_MAP_SWIZZLE_128B);
    CUtensorMap tk = tmap::make_kv_pages(k_cache, rows);
    CUtensorMap tv = tmap::make_kv_pages(v_cache, rows);
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(pf::prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, pf::SMEM);
      attr = true;
    }
    if (launch_pdl(pf::prefill_kernel, dim3(num_tiles * Hq), dim3(pf::kThreads), pf::SMEM, st, tq,
                   tk, tv, p) != cudaSuccess)
      return -4;
  } catch (const std::exception &) {
    return -3;
  }
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}
