// kv_tier.cu -- page moves between the device KV pool and a pinned host pool.
//
// Both pools have the layout [layers][pages][heads][16][128] (bf16) for K and
// for V, so a page of one layer is one contiguous run of heads*16*128*2
// bytes in either pool. The host pool is pinned memory, which unified
// addressing maps into the device address space: the kernel reads (fetch)
// or writes (spill) it with ordinary 16-byte loads and stores that cross
// PCIe, one CTA per (page pair, layer, K|V) so that thousands of requests
// are in flight at once. Pairs are processed in the order given, which is
// the order the scheduling plane wants them available (most urgent first).
//
// The host pool may instead hold fp8 (e4m3) pages with one fp32 scale per
// (layer, page, head, K|V): a spill quantizes (amax / 448 over the head's
// 16 x 128 values), a fetch dequantizes into the bf16 staging pool. That
// halves the bytes crossing PCIe -- the bound of a tiered step once several
// GPUs share a host uplink -- at the cost of fp8 precision on cold pages.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "common.cuh"

namespace kvtier {

struct CopyArgs {
  const uint4 *src_k, *src_v;
  uint4 *dst_k, *dst_v;
  const int2 *pairs;  // (source page, destination page)
  int n_pairs;
  const int *n_dev;   // when set, the pair count is read here (graph-captured launches)
  int layers;
  long long src_layer_pages, dst_layer_pages;  // pages per layer in each pool
  int page_vec;       // 16-byte vectors per page of one layer
  int *status;        // a pair outside either pool is skipped and reported (kStatusBadIndex)
};

// A pair whose pages lie outside their pools is skipped; thread `lead`
// reports it. Uniform across the threads that share the pair.
__device__ __forceinline__ bool pair_ok(const int2 pr, long long src_pages, long long dst_pages, int *status,
                                        bool lead) {
  if (pr.x < 0 || pr.x >= src_pages) {
    if (lead) report_bad_index(status, kSiteCopySrcPage, pr.x);
    return false;
  }
  if (pr.y < 0 || pr.y >= dst_pages) {
    if (lead) report_bad_index(status, kSiteCopyDstPage, pr.y);
    return false;
  }
  return true;
}

__global__ void __launch_bounds__(256) page_copy_kernel(const CopyArgs a) {
  // units (pair, layer, k|v), pair slowest, grid-stride: a fixed grid serves
  // any count (the count may only be known on the device)
  const int per_pair = 2 * a.layers;
  const int n = a.n_dev != nullptr ? min(*a.n_dev, a.n_pairs) : a.n_pairs;
  const long long units = (long long)n * per_pair;
  for (long long u = blockIdx.x; u < units; u += gridDim.x) {
    const int pi = (int)(u / per_pair), rem = (int)(u % per_pair);
    const int layer = rem >> 1, kv = rem & 1;
    const int2 pr = a.pairs[pi];
    if (!pair_ok(pr, a.src_layer_pages, a.dst_layer_pages, a.status, threadIdx.x == 0)) continue;
    const uint4 *src = (kv ? a.src_v : a.src_k) + ((size_t)layer * a.src_layer_pages + pr.x) * a.page_vec;
    uint4 *dst = (kv ? a.dst_v : a.dst_k) + ((size_t)layer * a.dst_layer_pages + pr.y) * a.page_vec;
    // issue several loads before the stores: PCIe latency is microseconds
    constexpr int U = 4;
    for (int i0 = threadIdx.x; i0 < a.page_vec; i0 += blockDim.x * U) {
      uint4 v[U];
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const int i = i0 + k * blockDim.x;
        if (i < a.page_vec) v[k] = __ldcs(src + i);
      }
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const int i = i0 + k * blockDim.x;
        if (i < a.page_vec) __stcs(dst + i, v[k]);
      }
    }
  }
}

struct QuantArgs {
  const void *src_k, *src_v;
  void *dst_k, *dst_v;
  float *scale_k, *scale_v;  // the fp8 pool's scales, [layers][pages][heads]
  const int2 *pairs;         // (source page, destination page)
  int n_pairs;
  const int *n_dev;
  int layers, heads;
  long long src_layer_pages, dst_layer_pages;
  int to_fp8;                // 1: bf16 -> fp8 (spill), 0: fp8 -> bf16 (fetch)
  int *status;
};

constexpr int kHeadElems = 16 * 128;  // one page of one head

// 16 bf16 (two uint4) -> 16 fp8 (one uint4) times `inv`
__device__ __forceinline__ uint4 quant16(const uint4 a, const uint4 b, float inv) {
  const __nv_bfloat162 *h0 = reinterpret_cast<const __nv_bfloat162 *>(&a);
  const __nv_bfloat162 *h1 = reinterpret_cast<const __nv_bfloat162 *>(&b);
  uint4 out;
  uint16_t *o = reinterpret_cast<uint16_t *>(&out);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 f = __bfloat1622float2(h0[j]);
    o[j] = __nv_cvt_float2_to_fp8x2(make_float2(f.x * inv, f.y * inv), __NV_SATFINITE, __NV_E4M3);
    f = __bfloat1622float2(h1[j]);
    o[4 + j] = __nv_cvt_float2_to_fp8x2(make_float2(f.x * inv, f.y * inv), __NV_SATFINITE, __NV_E4M3);
  }
  return out;
}

// 16 fp8 (one uint4) times `scale` -> 16 bf16 (two uint4)
__device__ __forceinline__ void dequant16(const uint4 q, float scale, uint4 &a, uint4 &b) {
  const uint16_t *in = reinterpret_cast<const uint16_t *>(&q);
  __nv_bfloat162 *h0 = reinterpret_cast<__nv_bfloat162 *>(&a);
  __nv_bfloat162 *h1 = reinterpret_cast<__nv_bfloat162 *>(&b);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const __half2 hh(__nv_cvt_fp8x2_to_halfraw2(in[j], __NV_E4M3));
    const float2 f = __half22float2(hh);
    const __nv_bfloat162 r = __floats2bfloat162_rn(f.x * scale, f.y * scale);
    if (j < 4) h0[j] = r; else h1[j - 4] = r;
  }
}

// One warp per (pair, layer, K|V, head) unit, grid-stride over all warps.
// Lane l owns 16-element groups l, l + 32, l + 64, l + 96 of the head's 2048
// values: 64 B of fp8 / 128 B of bf16 per group set, all loads in flight
// before any store.
__global__ void __launch_bounds__(256) quant_copy_kernel(const QuantArgs a) {
  const int lane = threadIdx.x & 31;
  const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long warps = ((long long)gridDim.x * blockDim.x) >> 5;
  const int n = a.n_dev != nullptr ? min(*a.n_dev, a.n_pairs) : a.n_pairs;
  const int per_pair = 2 * a.layers * a.heads;
  const long long units = (long long)n * per_pair;
  for (long long u = warp; u < units; u += warps) {
    const int pi = (int)(u / per_pair);
    int rem = (int)(u % per_pair);
    const int head = rem % a.heads;
    rem /= a.heads;
    const int kv = rem & 1, layer = rem >> 1;
    const int2 pr = a.pairs[pi];
    if (!pair_ok(pr, a.src_layer_pages, a.dst_layer_pages, a.status, lane == 0)) continue;
    const size_t src_head = ((size_t)layer * a.src_layer_pages + pr.x) * a.heads + head;
    const size_t dst_head = ((size_t)layer * a.dst_layer_pages + pr.y) * a.heads + head;
    if (a.to_fp8) {
      const uint4 *src = static_cast<const uint4 *>(kv ? a.src_v : a.src_k) + src_head * (kHeadElems / 8);
      uint4 *dst = static_cast<uint4 *>(kv ? a.dst_v : a.dst_k) + dst_head * (kHeadElems / 16);
      uint4 x[8];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        x[2 * g] = __ldcs(src + 2 * (lane + 32 * g));
        x[2 * g + 1] = __ldcs(src + 2 * (lane + 32 * g) + 1);
      }
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&x[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h[j]);
          amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float scale = amax > 0.f ? amax / 448.f : 1.f;
      const float inv = 1.f / scale;
#pragma unroll
      for (int g = 0; g < 4; ++g) __stcs(dst + lane + 32 * g, quant16(x[2 * g], x[2 * g + 1], inv));
      if (lane == 0) (kv ? a.scale_v : a.scale_k)[dst_head] = scale;
    } else {
      const uint4 *src = static_cast<const uint4 *>(kv ? a.src_v : a.src_k) + src_head * (kHeadElems / 16);
      uint4 *dst = static_cast<uint4 *>(kv ? a.dst_v : a.dst_k) + dst_head * (kHeadElems / 8);
      uint4 q[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) q[g] = __ldcs(src + lane + 32 * g);
      const float scale = (kv ? a.scale_v : a.scale_k)[src_head];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint4 lo, hi;
        dequant16(q[g], scale, lo, hi);
        __stcs(dst + 2 * (lane + 32 * g), lo);
        __stcs(dst + 2 * (lane + 32 * g) + 1, hi);
      }
    }
  }
}

}  // namespace kvtier

// Copy page data (all layers, K and V) for every (src, dst) pair from pool A
// to pool B. Pools are [layers][pages_A|B][heads][16][128] bf16; either may be
// pinned host memory. With `n_dev`, `n_pairs` is the capacity and the count
// actually copied is read from *n_dev on the device. A pair naming a page
// outside its pool is skipped and reported in `status` (kStatusBadIndex).
// Returns 0, -1 on bad arguments, -4 on a launch error.
extern "C" int sched_kv_page_copy(const void *src_k, const void *src_v, long long src_pages, void *dst_k,
                                  void *dst_v, long long dst_pages, const int32_t *pairs, int n_pairs,
                                  const int *n_dev, int layers, int heads, int *status, cudaStream_t st) {
  if (n_pairs <= 0) return 0;
  if (layers <= 0 || heads <= 0 || src_pages <= 0 || dst_pages <= 0) return -1;
  kvtier::CopyArgs a{};
  a.src_k = static_cast<const uint4 *>(src_k);
  a.src_v = static_cast<const uint4 *>(src_v);
  a.dst_k = static_cast<uint4 *>(dst_k);
  a.dst_v = static_cast<uint4 *>(dst_v);
  a.pairs = reinterpret_cast<const int2 *>(pairs);
  a.n_pairs = n_pairs;
  a.n_dev = n_dev;
  a.layers = layers;
  a.src_layer_pages = src_pages;
  a.dst_layer_pages = dst_pages;
  a.page_vec = heads * 16 * 128 * 2 / 16;
  a.status = status;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long units = (long long)n_pairs * 2 * layers;
  const int grid = (int)std::min<long long>(units, (long long)sms * 8);
  kvtier::page_copy_kernel<<<grid, 256, 0, st>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

// Page moves between a bf16 pool and an fp8 pool (to_fp8 = 1: bf16 source,
// fp8 destination; 0: the reverse). `scale_k` / `scale_v` belong to the fp8
// pool ([layers][its pages][heads] fp32): written by a spill, read by a
// fetch. Pairs and `n_dev` as for sched_kv_page_copy.
extern "C" int sched_kv_page_copy_fp8(const void *src_k, const void *src_v, long long src_pages, void *dst_k,
                                      void *dst_v, long long dst_pages, float *scale_k, float *scale_v, int to_fp8,
                                      const int32_t *pairs, int n_pairs, const int *n_dev, int layers, int heads,
                                      int *status, cudaStream_t st) {
  if (n_pairs <= 0) return 0;
  if (layers <= 0 || heads <= 0 || src_pages <= 0 || dst_pages <= 0 || !scale_k || !scale_v) return -1;
  kvtier::QuantArgs a{};
  a.src_k = src_k;
  a.src_v = src_v;
  a.dst_k = dst_k;
  a.dst_v = dst_v;
  a.scale_k = scale_k;
  a.scale_v = scale_v;
  a.pairs = reinterpret_cast<const int2 *>(pairs);
  a.n_pairs = n_pairs;
  a.n_dev = n_dev;
  a.layers = layers;
  a.heads = heads;
  a.src_layer_pages = src_pages;
  a.dst_layer_pages = dst_pages;
  a.to_fp8 = to_fp8 ? 1 : 0;
  a.status = status;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long warps = (long long)n_pairs * 2 * layers * heads;
  const int grid = (int)std::min<long long>((warps + 7) / 8, (long long)sms * 8);
  kvtier::quant_copy_kernel<<<grid, 256, 0, st>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}
