// elementwise.cu -- the bandwidth-bound per-token kernels of a decoder layer.
//
//   * fused residual-add + RMSNorm: res += x; y = res * rsqrt(mean(res^2) + eps) * w
//     (one read of x and res, one write of res and y: the add that closes a
//     sub-block and the norm that opens the next one cost one pass);
//   * RoPE + KV append: rotates q and k of the fused QKV projection output,
//     writes q to the attention input and k, v straight into their pages of
//     the paged cache (no intermediate k/v tensors);
//   * token embedding gather;
//   * greedy sampling (row argmax over the vocabulary);
//   * the sequence-parallel norm of the tensor-parallel layer: reduction of
//     the world's row partials (pushed by the reduce-scatter GEMM), residual
//     add + RMSNorm with the same arithmetic as the fused add + RMSNorm, and
//     the all-gather push of the normed row to every rank.
// All accesses are 16-byte vectors; one CTA per token row.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "sched/ptx.cuh"
#include "sp_api.h"

namespace ew {

template <int NT>
__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) s += red[i];
  return s;
}

// H = hidden size, multiple of 8; NT threads, each owns H / NT / 8 vectors.
template <int NT, int VPT>
__global__ void __launch_bounds__(NT) add_rmsnorm_kernel(const __nv_bfloat16 *__restrict__ x,
                                                         __nv_bfloat16 *__restrict__ res,
                                                         const __nv_bfloat16 *__restrict__ w,
                                                         __nv_bfloat16 *__restrict__ y, int H,
                                                         float eps) {
  __shared__ float red[NT / 32];
  const size_t row = blockIdx.x;
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * NT) * 8;
    if (c < H) {
      uint4 xv = *reinterpret_cast<const uint4 *>(x + row * H + c);
      const __nv_bfloat16 *xe = reinterpret_cast<const __nv_bfloat16 *>(&xv);
      if (res != nullptr) {
        uint4 rv = *reinterpret_cast<const uint4 *>(res + row * H + c);
        const __nv_bfloat16 *re = reinterpret_cast<const __nv_bfloat16 *>(&rv);
        uint4 ov;
        __nv_bfloat16 *oe = reinterpret_cast<__nv_bfloat16 *>(&ov);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          // the residual stream is kept in bf16: round the sum once, like a
          // separate add kernel would
          oe[j] = __float2bfloat16(__bfloat162float(xe[j]) + __bfloat162float(re[j]));
          v[i][j] = __bfloat162float(oe[j]);
        }
        *reinterpret_cast<uint4 *>(res + row * H + c) = ov;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = __bfloat162float(xe[j]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  const float inv = rsqrtf(block_sum<NT>(ss, red) / (float)H + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * NT) * 8;
    if (c < H) {
      uint4 wv = *reinterpret_cast<const uint4 *>(w + c);
      const __nv_bfloat16 *we = reinterpret_cast<const __nv_bfloat16 *>(&wv);
      uint4 ov;
      ov.x = pack_bf16x2(v[i][0] * inv * __bfloat162float(we[0]), v[i][1] * inv * __bfloat162float(we[1]));
      ov.y = pack_bf16x2(v[i][2] * inv * __bfloat162float(we[2]), v[i][3] * inv * __bfloat162float(we[3]));
      ov.z = pack_bf16x2(v[i][4] * inv * __bfloat162float(we[4]), v[i][5] * inv * __bfloat162float(we[5]));
      ov.w = pack_bf16x2(v[i][6] * inv * __bfloat162float(we[6]), v[i][7] * inv * __bfloat162float(we[7]));
      *reinterpret_cast<uint4 *>(y + row * H + c) = ov;
    }
  }
}

// One warp per head of one token. Rotate-half RoPE (pairs d, d + D/2) with a
// precomputed [max_pos, D/2] table of (cos, sin). Head order in qkv:
// Hq query heads, Hkv key heads, Hkv value heads.
template <int D>
__global__ void rope_kv_append_kernel(const __nv_bfloat16 *__restrict__ qkv,
                                      const int32_t *__restrict__ pos,
                                      const int32_t *__restrict__ slot,
                                      const float2 *__restrict__ cos_sin,
                                      __nv_bfloat16 *__restrict__ q_out,
                                      __nv_bfloat16 *__restrict__ k_cache,
                                      __nv_bfloat16 *__restrict__ v_cache, int Hq, int Hkv,
                                      int page_size, int num_pages, int *status) {
  constexpr int HALF = D / 2;
  const int t = blockIdx.x;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nheads = Hq + 2 * Hkv;
  const int p = pos[t];
  int s = slot[t];
  // a slot outside the cache is reported and its cache writes skipped
  if (s >= 0 && (long long)s >= (long long)num_pages * page_size) {
    if (threadIdx.x == 0) report_bad_index(status, kSiteKvSlot, s);
    s = -1;
  }
  const int page = s / page_size, off = s % page_size;
  const __nv_bfloat16 *src_row = qkv + (size_t)t * nheads * D;
  for (int h = warp; h < nheads; h += blockDim.x / 32) {
    const __nv_bfloat16 *src = src_row + (size_t)h * D;
    __nv_bfloat16 *dst;
    if (h < Hq) {
      dst = q_out + ((size_t)t * Hq + h) * D;
    } else if (h < Hq + Hkv) {
      if (s < 0) continue;  // padding token: no cache write
      dst = k_cache + (((size_t)page * Hkv + (h - Hq)) * page_size + off) * D;
    } else {
      if (s < 0) continue;
      dst = v_cache + (((size_t)page * Hkv + (h - Hq - Hkv)) * page_size + off) * D;
      // value heads are copied unrotated
      for (int d = lane * 8; d < D; d += 32 * 8)
        *reinterpret_cast<uint4 *>(dst + d) = *reinterpret_cast<const uint4 *>(src + d);
      continue;
    }
    // each lane rotates pairs (d, d + HALF) for d = lane, lane + 32, ...
    for (int d = lane; d < HALF; d += 32) {
      const float2 cs = cos_sin[(size_t)p * HALF + d];
      const float a = __bfloat162float(src[d]);
      const float b = __bfloat162float(src[d + HALF]);
      dst[d] = __float2bfloat16(a * cs.x - b * cs.y);
      dst[d + HALF] = __float2bfloat16(b * cs.x + a * cs.y);
    }
  }
}

// A negative id -(1 + j) with `prev` given names row j of `prev`: a token the
// previous step sampled and that is still only on the device (the engine
// plans step k + 1 before step k's tokens reach the host).
__global__ void embedding_kernel(const int32_t *__restrict__ ids, const int32_t *__restrict__ prev,
                                 int n_prev, const __nv_bfloat16 *__restrict__ table,
                                 __nv_bfloat16 *__restrict__ out, int H, int vocab, int *status) {
  const int t = blockIdx.x;
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  int id = ids[t];
  if (id < 0 && prev != nullptr && -(id + 1) < n_prev) id = prev[-(id + 1)];
  if (id < 0 || id >= vocab) {  // reported; the row is zeroed instead of read out of bounds
    if (threadIdx.x == 0) report_bad_index(status, kSiteTokenId, id);
    for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8)
      *reinterpret_cast<uint4 *>(out + (size_t)t * H + c) = make_uint4(0, 0, 0, 0);
    return;
  }
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8)
    *reinterpret_cast<uint4 *>(out + (size_t)t * H + c) =
        *reinterpret_cast<const uint4 *>(table + (size_t)id * H + c);
}

// Vocabulary-parallel greedy sampling across tensor-parallel ranks, inside
// the argmax kernel: each row's (max, global id) goes to every rank as one
// 16-byte line {max bits, epoch, id, epoch} (an 8-byte half lands whole), and
// the row's block then polls the world's lines for that row in its own buffer
// and keeps the largest value, the lowest id on ties. `state` = this rank's
// [epoch, done]: a call uses epoch + 1 and the buffer set of its parity; the
// last block advances the epoch (0 skipped on wrap-around). world == 0: off.
struct ArgmaxExchange {
  uint4 *lines[8];     // every rank's line buffer: 2 sets x [world][rows] lines
  int world, rank;
  uint32_t *state;     // this rank's [epoch, done] (device, zero at start)
  long long set_lines;  // lines per set (>= world x rows)
  int *status;
};

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void exchange_row(const ArgmaxExchange &x, int t, int rows, float &best, int &gid) {
  const uint32_t e = ld_volatile_u32(x.state) + 1u;
  const size_t set = (size_t)(e & 1u) * x.set_lines;
  const size_t mine = set + (size_t)x.rank * rows + t;
  for (int j = 0; j < x.world; ++j)
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(x.lines[j] + mine),
                 "r"(__float_as_uint(best)), "r"(e), "r"((uint32_t)gid), "r"(e)
                 : "memory");
  float b = -INFINITY;
  int g = 0x7fffffff;
  for (int src = 0; src < x.world; ++src) {
    const uint4 *q = x.lines[x.rank] + set + (size_t)src * rows + t;
    uint4 l = make_uint4(0, 0, 0, 0);
    const uint64_t start = ptx::globaltimer_ns();
    for (uint32_t polls = 0;; ++polls) {
      asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(l.x), "=r"(l.y), "=r"(l.z), "=r"(l.w)
                   : "l"(q)
                   : "memory");
      if (l.y == e && l.w == e) break;
      if ((polls & 63u) == 63u && ptx::globaltimer_ns() - start > kWaitBudgetNs) {
        report_status(x.status, kStatusPeerTimeout);
        break;
      }
    }
    const float v = __uint_as_float(l.x);
    const int i = (int)l.z;
    if (v > b || (v == b && i < g)) {
      b = v;
      g = i;
    }
  }
  best = b;
  gid = g;
}

// Row argmax; ties resolve to the lowest index. Also emits the row max so a
// vocabulary-parallel caller can combine shards (value, index) pairs; with
// an exchange (ArgmaxExchange::world > 0) the shards are combined here.
__global__ void __launch_bounds__(1024) argmax_kernel(const __nv_bfloat16 *__restrict__ logits,
                                                      int V, int ld, int32_t *__restrict__ ids,
                                                      float *__restrict__ maxv, int id_offset,
                                                      const ArgmaxExchange x) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const int t = blockIdx.x;
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const __nv_bfloat16 *row = logits + (size_t)t * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  // 16-byte vector loads only where the row starts on a 16-byte boundary
  // (a row pitch that is not a multiple of 8 elements, e.g. a vocabulary
  // shard of odd width, takes the scalar loop for the whole row)
  const bool vec = (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
  const int nvec = vec ? V / 8 : 0;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    uint4 u = *reinterpret_cast<const uint4 *>(row + i * 8);
    const __nv_bfloat16 *e = reinterpret_cast<const __nv_bfloat16 *>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = __bfloat162float(e[j]);
      if (v > best) {
        best = v;
        bi = i * 8 + j;
      }
    }
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += blockDim.x) {
    const float v = __bfloat162float(row[i]);
    if (v > best) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    best = l < (int)(blockDim.x / 32) ? sv[l] : -INFINITY;
    bi = l < (int)(blockDim.x / 32) ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (l == 0) {
      int gid = bi + id_offset;
      if (x.world > 0) exchange_row(x, t, gridDim.x, best, gid);
      ids[t] = gid;
      if (maxv != nullptr) maxv[t] = best;
      if (x.world > 0) {
        __threadfence();
        if (atomicAdd(x.state + 1, 1u) == gridDim.x - 1) {  // the call's last block
          x.state[1] = 0u;
          const uint32_t e = ld_volatile_u32(x.state) + 1u;
          __threadfence();
          x.state[0] = e == 0xFFFFFFFFu ? 1u : e;
        }
      }
    }
  }
}

// Sequence-parallel norm: one CTA per owned row t. The arithmetic after the
// reduction is add_rmsnorm_kernel's, with the same NT / VPT, so the normed
// rows are bit-identical to those of the all-reduce path.
template <int NT, int VPT>
__global__ void __launch_bounds__(NT) sp_reduce_norm_kernel(const SpNormArgs a) {
  __shared__ float red[NT / 32];
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  for (int i = blockIdx.x * NT + threadIdx.x; i < a.clear_n; i += gridDim.x * NT) a.clear[i] = 0u;
  const int t = sp_row_begin(a.rank, a.T, a.world) + (int)blockIdx.x;
  if (t >= sp_row_begin(a.rank + 1, a.T, a.world)) return;  // a rank without rows clears only
  const int H = a.H;
  const int nflags = a.world * (H / 128);
  // every source rank's every 128-column tile of the row has landed
  for (int i = threadIdx.x; i < nflags; i += NT) {
    const uint32_t *f = a.row_flags + (size_t)i * a.T + t;
    if (ptx::ld_acquire_sys(f) == 0u) {
      const uint64_t start = ptx::globaltimer_ns();
      bool ok = false;
      while (!ok) {
        for (int k = 0; k < 64 && !ok; ++k) ok = ptx::ld_acquire_sys(f) != 0u;
        if (!ok && ptx::globaltimer_ns() - start > kWaitBudgetNs) break;
      }
      if (!ok) report_status(a.status, kStatusPeerTimeout);
    }
  }
  __syncthreads();
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * NT) * 8;
    if (c < H) {
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      for (int src = 0; src < a.world; ++src) {  // rank order: the same sum on every rank
        const uint4 u = __ldcv(reinterpret_cast<const uint4 *>(a.slab + ((size_t)src * a.T + t) * H + c));
        const __nv_bfloat16 *e = reinterpret_cast<const __nv_bfloat16 *>(&u);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += __bfloat162float(e[j]);
      }
      uint4 dv;
      dv.x = pack_bf16x2(acc[0], acc[1]);
      dv.y = pack_bf16x2(acc[2], acc[3]);
      dv.z = pack_bf16x2(acc[4], acc[5]);
      dv.w = pack_bf16x2(acc[6], acc[7]);
      if (a.delta != nullptr) *reinterpret_cast<uint4 *>(a.delta + (size_t)t * H + c) = dv;
      const __nv_bfloat16 *xe = reinterpret_cast<const __nv_bfloat16 *>(&dv);
      const uint4 rv = *reinterpret_cast<const uint4 *>(a.res + (size_t)t * H + c);
      const __nv_bfloat16 *re = reinterpret_cast<const __nv_bfloat16 *>(&rv);
      uint4 ov;
      __nv_bfloat16 *oe = reinterpret_cast<__nv_bfloat16 *>(&ov);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        oe[j] = __float2bfloat16(__bfloat162float(xe[j]) + __bfloat162float(re[j]));
        v[i][j] = __bfloat162float(oe[j]);
      }
      *reinterpret_cast<uint4 *>(a.res + (size_t)t * H + c) = ov;
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  const float inv = rsqrtf(block_sum<NT>(ss, red) / (float)H + a.eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * NT) * 8;
    if (c < H) {
      uint4 wv = *reinterpret_cast<const uint4 *>(a.w + c);
      const __nv_bfloat16 *we = reinterpret_cast<const __nv_bfloat16 *>(&wv);
      uint4 ov;
      ov.x = pack_bf16x2(v[i][0] * inv * __bfloat162float(we[0]), v[i][1] * inv * __bfloat162float(we[1]));
      ov.y = pack_bf16x2(v[i][2] * inv * __bfloat162float(we[2]), v[i][3] * inv * __bfloat162float(we[3]));
      ov.z = pack_bf16x2(v[i][4] * inv * __bfloat162float(we[4]), v[i][5] * inv * __bfloat162float(we[5]));
      ov.w = pack_bf16x2(v[i][6] * inv * __bfloat162float(we[6]), v[i][7] * inv * __bfloat162float(we[7]));
      for (int j = 0; j < a.world; ++j)  // all-gather: NVLink stores into every rank's copy
        *reinterpret_cast<uint4 *>(a.gather[j] + (size_t)t * H + c) = ov;
    }
  }
  __threadfence_system();
  __syncthreads();
  if ((int)threadIdx.x < a.world) ptx::st_release_sys(a.ready[threadIdx.x] + t, 1u);
  // the row's partials are consumed: its flags are zero for the slab set's next use
  for (int i = threadIdx.x; i < nflags; i += NT) a.row_flags[(size_t)i * a.T + t] = 0u;
}

__global__ void __launch_bounds__(256) sp_wait_rows_kernel(const uint32_t *ready, int T, int *status) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    if (ptx::ld_acquire_sys(ready + t) != 0u) continue;
    const uint64_t start = ptx::globaltimer_ns();
    bool ok = false;
    while (!ok) {
      for (int k = 0; k < 64 && !ok; ++k) ok = ptx::ld_acquire_sys(ready + t) != 0u;
      if (!ok && ptx::globaltimer_ns() - start > kWaitBudgetNs) break;
    }
    if (!ok) report_status(status, kStatusPeerTimeout);
  }
  __syncthreads();
}

}  // namespace ew

extern "C" int sched_add_rmsnorm(const void *x, void *res, const void *w, void *y, int T, int H,
                                 float eps, cudaStream_t st) {
  if (T <= 0) return 0;
  if (H % 8 != 0) return -1;
  const __nv_bfloat16 *xb = static_cast<const __nv_bfloat16 *>(x);
  __nv_bfloat16 *rb = static_cast<__nv_bfloat16 *>(res);
  const __nv_bfloat16 *wb = static_cast<const __nv_bfloat16 *>(w);
  __nv_bfloat16 *yb = static_cast<__nv_bfloat16 *>(y);
  if (H <= 256 * 8 * 2)
    launch_pdl(ew::add_rmsnorm_kernel<256, 2>, T, 256, 0, st, xb, rb, wb, yb, H, eps);
  else if (H <= 512 * 8 * 2)
    launch_pdl(ew::add_rmsnorm_kernel<512, 2>, T, 512, 0, st, xb, rb, wb, yb, H, eps);
  else if (H <= 1024 * 8 * 2)
    launch_pdl(ew::add_rmsnorm_kernel<1024, 2>, T, 1024, 0, st, xb, rb, wb, yb, H, eps);
  else
    return -1;
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int sched_rope_kv_append(const void *qkv, const int32_t *pos, const int32_t *slot,
                                    const float *cos_sin, void *q_out, void *k_cache,
                                    void *v_cache, int T, int Hq, int Hkv, int D, int page_size,
                                    int num_pages, int *status, cudaStream_t st) {
  if (T <= 0) return 0;
  if (D != 128) return -1;
  ew::rope_kv_append_kernel<128><<<T, 256, 0, st>>>(
      static_cast<const __nv_bfloat16 *>(qkv), pos, slot, reinterpret_cast<const float2 *>(cos_sin),
      static_cast<__nv_bfloat16 *>(q_out), static_cast<__nv_bfloat16 *>(k_cache),
      static_cast<__nv_bfloat16 *>(v_cache), Hq, Hkv, page_size, num_pages, status);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int sched_embedding(const int32_t *ids, const int32_t *prev, int n_prev, const void *table, void *out,
                               int T, int H, int vocab, int *status, cudaStream_t st) {
  if (T <= 0) return 0;
  // 16-byte row copies: rows of a multiple of 8 bf16 on 16-byte-aligned bases
  if (H % 8 != 0 || (reinterpret_cast<uintptr_t>(table) & 15u) != 0 || (reinterpret_cast<uintptr_t>(out) & 15u) != 0)
    return -1;
  launch_pdl(ew::embedding_kernel, T, 256, 0, st, ids, prev, prev != nullptr ? n_prev : 0,
             static_cast<const __nv_bfloat16 *>(table), static_cast<__nv_bfloat16 *>(out), H, vocab, status);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int sched_argmax(const void *logits, int T, int V, int ld, int32_t *ids, float *maxv,
                            int id_offset, cudaStream_t st) {
  if (T <= 0) return 0;
  ew::ArgmaxExchange none{};
  launch_pdl(ew::argmax_kernel, T, 1024, 0, st, static_cast<const __nv_bfloat16 *>(logits), V, ld,
             ids, maxv, id_offset, none);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

// Vocabulary-parallel argmax with the ranks' (max, id) exchange in the same
// kernel: lines[j] is rank j's line buffer (two sets of set_lines 16-byte
// lines, set_lines >= world * T), state this rank's [epoch, done] pair.
extern "C" int sched_argmax_exchange(const void *logits, int T, int V, int ld, int32_t *ids, float *maxv,
                                     int id_offset, void *const *lines, int world, int rank, uint32_t *state,
                                     long long set_lines, int *status, cudaStream_t st) {
  if (T <= 0) return 0;
  if (world < 1 || world > 8 || rank < 0 || rank >= world || state == nullptr || set_lines < (long long)world * T)
    return -1;
  ew::ArgmaxExchange x{};
  for (int j = 0; j < world; ++j) {
    if (lines[j] == nullptr || (reinterpret_cast<uintptr_t>(lines[j]) & 15) != 0) return -1;
    x.lines[j] = static_cast<uint4 *>(lines[j]);
  }
  x.world = world;
  x.rank = rank;
  x.state = state;
  x.set_lines = set_lines;
  x.status = status;
  launch_pdl(ew::argmax_kernel, T, 1024, 0, st, static_cast<const __nv_bfloat16 *>(logits), V, ld,
             ids, maxv, id_offset, x);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int sched_sp_reduce_norm(const SpNormArgs *args, cudaStream_t st) {
  if (args == nullptr) return -1;
  const SpNormArgs &a = *args;
  if (a.T <= 0) return 0;
  if (a.H % 128 != 0 || a.world < 1 || a.world > kMaxWorld || a.rank < 0 || a.rank >= a.world) return -1;
  if (a.slab == nullptr || a.row_flags == nullptr || a.res == nullptr || a.w == nullptr) return -1;
  for (int j = 0; j < a.world; ++j)
    if (a.gather[j] == nullptr || a.ready[j] == nullptr) return -1;
  if (a.clear_n > 0 && a.clear == nullptr) return -1;
  const int rows = sp_row_begin(a.rank + 1, a.T, a.world) - sp_row_begin(a.rank, a.T, a.world);
  const int grid = rows > 0 ? rows : 1;
  // the thread shapes of sched_add_rmsnorm (same reduction order)
  if (a.H <= 256 * 8 * 2)
    launch_pdl(ew::sp_reduce_norm_kernel<256, 2>, grid, 256, 0, st, a);
  else if (a.H <= 512 * 8 * 2)
    launch_pdl(ew::sp_reduce_norm_kernel<512, 2>, grid, 512, 0, st, a);
  else if (a.H <= 1024 * 8 * 2)
    launch_pdl(ew::sp_reduce_norm_kernel<1024, 2>, grid, 1024, 0, st, a);
  else
    return -1;
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int sched_sp_wait_rows(const uint32_t *ready, int T, int *status, cudaStream_t st) {
  if (T <= 0) return 0;
  if (ready == nullptr) return -1;
  launch_pdl(ew::sp_wait_rows_kernel, 1, 256, 0, st, ready, T, status);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}
