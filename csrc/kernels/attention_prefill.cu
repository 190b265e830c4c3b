// attention_prefill.cu -- causal attention of prefill chunks over the paged KV cache.
//
// Each CTA owns 64 query rows of one request and one query head (4 warps x
// 16 rows) and streams that request's KV pages in 64-token tiles through a
// double-buffered cp.async ring. QK^T and PV use the warp-level bf16 MMA
// (m16n8k16) with the online softmax kept in registers (the FlashAttention-2
// schedule). The query rows are the newest tokens of the request: row i has
// absolute position q_pos0 + i and sees KV tokens [0, q_pos0 + i], which
// covers both a whole prompt and a chunk appended to a cached prefix.
//
// Prefill attention is ~3% of a 1536-token prefill's FLOPs on Llama-3-8B (the
// projections dominate and run on tcgen05, gemm.cu); this kernel is the
// warp-MMA version of it.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"

namespace pf {

constexpr int D = 128;
constexpr int BQ = 64;
constexpr int BKV = 64;
constexpr int PITCH = D + 8;  // padded smem row (elements): conflict-free ldmatrix
constexpr int kThreads = 128;

struct QTile {
  int32_t req;     // request index (row of block table / kv_lens)
  int32_t q_row0;  // first row of this tile in the packed q / out tensors
  int32_t nq;      // rows in this tile (<= 64)
  int32_t q_pos0;  // absolute position of the first row
};

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool pred) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int n = pred ? 16 : 0;  // zero-fill when out of range
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(kThreads) prefill_kernel(
    const __nv_bfloat16 *__restrict__ q, __nv_bfloat16 *__restrict__ out,
    const __nv_bfloat16 *__restrict__ k_cache, const __nv_bfloat16 *__restrict__ v_cache,
    const int32_t *__restrict__ block_table, int bt_stride, const int32_t *__restrict__ kv_lens,
    const QTile *__restrict__ tiles, int Hq, int Hkv, int page_size, float scale_log2) {
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16 *sQ = reinterpret_cast<__nv_bfloat16 *>(smem);
  __nv_bfloat16 *sK = sQ + BQ * PITCH;        // [2][BKV][PITCH]
  __nv_bfloat16 *sV = sK + 2 * BKV * PITCH;   // [2][BKV][PITCH]

  const QTile tile = tiles[blockIdx.x];
  const int hq = blockIdx.y;
  const int kvh = hq / (Hq / Hkv);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int kv_len = kv_lens[tile.req];
  const int32_t *bt = block_table + (size_t)tile.req * bt_stride;
  const int kv_stop = min(kv_len, tile.q_pos0 + tile.nq);  // last row sees [0, q_pos0+nq-1]
  const int ntiles = (kv_stop + BKV - 1) / BKV;

  // Q tile -> smem (rows beyond nq zero)
  for (int i = tid; i < BQ * (D / 8); i += kThreads) {
    const int r = i / (D / 8), c = (i % (D / 8)) * 8;
    const bool ok = r < tile.nq;
    const __nv_bfloat16 *src = q + ((size_t)(tile.q_row0 + (ok ? r : 0)) * Hq + hq) * D + c;
    cp_async16(sQ + r * PITCH + c, src, ok);
  }
  auto load_kv = [&](int kt, int buf) {
    for (int i = tid; i < BKV * (D / 8); i += kThreads) {
      const int r = i / (D / 8), c = (i % (D / 8)) * 8;
      const int tok = kt * BKV + r;
      const bool ok = tok < kv_stop;
      const int page = ok ? bt[tok / page_size] : 0;
      const size_t off = (((size_t)page * Hkv + kvh) * page_size + (ok ? tok % page_size : 0)) * D + c;
      cp_async16(sK + (buf * BKV + r) * PITCH + c, k_cache + off, ok);
      cp_async16(sV + (buf * BKV + r) * PITCH + c, v_cache + off, ok);
    }
  };
  if (ntiles > 0) load_kv(0, 0);
  cp_async_commit();

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  const int g = lane / 4, tq = lane % 4;
  const int row0 = warp * 16 + g;  // this thread's rows: row0, row0 + 8
  const int qp0 = tile.q_pos0 + row0, qp1 = qp0 + 8;
  uint32_t qa[D / 16][4];

  for (int kt = 0; kt < ntiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ntiles) load_kv(kt + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kt == 0) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        ldsm_x4(qa[kk], sQ + (warp * 16 + (lane % 16)) * PITCH + kk * 16 + (lane / 16) * 8);
    }
    const __nv_bfloat16 *kb = sK + buf * BKV * PITCH;
    const __nv_bfloat16 *vb = sV + buf * BKV * PITCH;
    float s[BKV / 8][4];
#pragma unroll
    for (int n = 0; n < BKV / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int n2 = 0; n2 < BKV / 16; ++n2) {
        uint32_t b[4];
        ldsm_x4(b, kb + (n2 * 16 + (lane % 8) + (lane / 16) * 8) * PITCH + kk * 16 +
                       ((lane / 8) % 2) * 8);
        mma16816(s[2 * n2], qa[kk], b[0], b[1]);
        mma16816(s[2 * n2 + 1], qa[kk], b[2], b[3]);
      }
    }
    // mask + online softmax (rows row0 and row0 + 8)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < BKV / 8; ++n) {
      const int c0 = kt * BKV + n * 8 + 2 * tq;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = c0 + (e & 1);
        const int qp = (e < 2) ? qp0 : qp1;
        const bool ok = col <= qp && col < kv_stop;
        s[n][e] = ok ? s[n][e] * scale_log2 : -INFINITY;
        mx[e >> 1] = fmaxf(mx[e >> 1], s[n][e]);
      }
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mn = fmaxf(m[r], mx[r]);
      alpha[r] = (mn == -INFINITY) ? 1.f : exp2f(m[r] - mn);
      m[r] = mn;
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pa[BKV / 16][4];
#pragma unroll
    for (int n = 0; n < BKV / 8; ++n) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mr = m[e >> 1];
        pv[e] = (mr == -INFINITY) ? 0.f : exp2f(s[n][e] - mr);
        rs[e >> 1] += pv[e];
      }
      const int kk = n / 2, hi = n % 2;
      pa[kk][hi * 2 + 0] = pack_bf16x2(pv[0], pv[1]);
      pa[kk][hi * 2 + 1] = pack_bf16x2(pv[2], pv[3]);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l[r] = l[r] * alpha[r] + rs[r];
    }
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
    // P (A operand) x V: A fragment order is (row g k-lo, row g+8 k-lo, row g k-hi, row g+8 k-hi)
#pragma unroll
    for (int kk = 0; kk < BKV / 16; ++kk) {
      uint32_t a[4] = {pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3]};
#pragma unroll
      for (int n2 = 0; n2 < D / 16; ++n2) {
        uint32_t b[4];
        ldsm_x4_t(b, vb + (kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8) * PITCH + n2 * 16 +
                         (lane / 16) * 8);
        mma16816(o[2 * n2], a, b[0], b[1]);
        mma16816(o[2 * n2 + 1], a, b[2], b[3]);
      }
    }
    __syncthreads();
  }
  // write normalised rows
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = row0 + r * 8;
    if (row >= tile.nq) continue;
    const float inv = l[r] > 0.f ? 1.f / l[r] : 0.f;
    __nv_bfloat16 *dst = out + ((size_t)(tile.q_row0 + row) * Hq + hq) * D;
#pragma unroll
    for (int n = 0; n < D / 8; ++n)
      *reinterpret_cast<uint32_t *>(dst + n * 8 + 2 * tq) =
          pack_bf16x2(o[n][2 * r] * inv, o[n][2 * r + 1] * inv);
  }
}

}  // namespace pf

extern "C" int sched_attn_prefill(const void *q, void *out, const void *k_cache,
                                  const void *v_cache, const int32_t *block_table, int bt_stride,
                                  const int32_t *kv_lens, const void *tiles, int num_tiles, int Hq,
                                  int Hkv, int page_size, float sm_scale, cudaStream_t st) {
  if (num_tiles <= 0) return 0;
  const int smem = (pf::BQ + 4 * pf::BKV) * pf::PITCH * 2;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(pf::prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr = true;
  }
  pf::prefill_kernel<<<dim3(num_tiles, Hq), pf::kThreads, smem, st>>>(
      static_cast<const __nv_bfloat16 *>(q), static_cast<__nv_bfloat16 *>(out),
      static_cast<const __nv_bfloat16 *>(k_cache), static_cast<const __nv_bfloat16 *>(v_cache),
      block_table, bt_stride, kv_lens, static_cast<const pf::QTile *>(tiles), Hq, Hkv, page_size,
      sm_scale * 1.4426950408889634f);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}
