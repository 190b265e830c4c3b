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
#include <cuda_bf16.h>
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
};

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

}  // namespace kvtier

// Copy page data (all layers, K and V) for every (src, dst) pair from pool A
// to pool B. Pools are [layers][pages_A|B][heads][16][128] bf16; either may be
// pinned host memory. With `n_dev`, `n_pairs` is the capacity and the count
// actually copied is read from *n_dev on the device. Returns 0, -1 on bad
// arguments, -4 on a launch error.
extern "C" int sched_kv_page_copy(const void *src_k, const void *src_v, long long src_pages, void *dst_k,
                                  void *dst_v, long long dst_pages, const int32_t *pairs, int n_pairs,
                                  const int *n_dev, int layers, int heads, cudaStream_t st) {
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
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long units = (long long)n_pairs * 2 * layers;
  const int grid = (int)std::min<long long>(units, (long long)sms * 8);
  kvtier::page_copy_kernel<<<grid, 256, 0, st>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}
