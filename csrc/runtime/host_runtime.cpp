// host_runtime.cpp -- CPU-side runtime of the serving engine (C ABI, ctypes).
//
//   * page allocator: a LIFO free list of KV-cache pages (recently freed
//     pages are reused first, they are the likeliest to still sit in L2);
//   * decode planner: splits every decode request into S KV chunks of
//     128-token blocks and emits the work items the decode kernel consumes,
//     plus the merge table for split requests;
//   * orders: grouped LPT and the cluster-launch-control region order, the
//     same policies as the Python plane, for per-step use without Python
//     loops.
// Nothing here touches the GPU; it links only the C++ standard library.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <new>
#include <numeric>
#include <vector>

namespace {

struct PageAllocator {
  std::vector<int32_t> free_list;  // stack: back() is the next page handed out
  std::vector<uint8_t> in_use;
  explicit PageAllocator(int32_t n) : in_use(n, 0) {
    free_list.resize(n);
    for (int32_t i = 0; i < n; ++i) free_list[i] = n - 1 - i;  // page 0 first
  }
};

void grouped_lpt(const float *cost, int n, int block, int32_t *out) {
  if (block <= 1 || n <= block) {
    std::vector<int32_t> idx(n);
    std::iota(idx.begin(), idx.end(), 0);
    std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return cost[a] > cost[b]; });
    std::copy(idx.begin(), idx.end(), out);
    return;
  }
  const int nb = (n + block - 1) / block;
  std::vector<double> bc(nb, 0.0);
  for (int i = 0; i < n; ++i) bc[i / block] += cost[i];
  std::vector<int32_t> border(nb);
  std::iota(border.begin(), border.end(), 0);
  std::stable_sort(border.begin(), border.end(), [&](int a, int b) { return bc[a] > bc[b]; });
  int k = 0;
  for (int b : border)
    for (int i = b * block; i < std::min(n, (b + 1) * block); ++i) out[k++] = i;
}

}  // namespace

extern "C" {

void *sched_alloc_create(int32_t num_pages) {
  if (num_pages <= 0) return nullptr;
  return new (std::nothrow) PageAllocator(num_pages);
}

void sched_alloc_destroy(void *h) { delete static_cast<PageAllocator *>(h); }

int32_t sched_alloc_free_count(void *h) {
  return static_cast<int32_t>(static_cast<PageAllocator *>(h)->free_list.size());
}

// Take n pages into out[]; all or nothing. Returns 0, or -1 when short.
int32_t sched_alloc_take(void *h, int32_t n, int32_t *out) {
  auto *a = static_cast<PageAllocator *>(h);
  if (n < 0 || (size_t)n > a->free_list.size()) return -1;
  for (int32_t i = 0; i < n; ++i) {
    int32_t p = a->free_list.back();
    a->free_list.pop_back();
    a->in_use[p] = 1;
    out[i] = p;
  }
  return 0;
}

// Return pages; a page that is not in use (double free) is rejected: -1.
int32_t sched_alloc_give(void *h, int32_t n, const int32_t *pages) {
  auto *a = static_cast<PageAllocator *>(h);
  for (int32_t i = 0; i < n; ++i) {
    const int32_t p = pages[i];
    if (p < 0 || (size_t)p >= a->in_use.size() || !a->in_use[p]) return -1;
  }
  for (int32_t i = 0; i < n; ++i) {
    a->in_use[pages[i]] = 0;
    a->free_list.push_back(pages[i]);
  }
  return 0;
}

// Decode work items for B requests split S ways (S >= 1).
//   items[4 * (b * S + s)] = {b, begin, end, part}; begin is a multiple of
//   `blk`; empty chunks have begin == end. With S == 1, part = -1 (the kernel
//   writes the final output) and no merge rows are emitted; otherwise part =
//   b * S + s and merge_begin[b] = b * S (B + 1 entries), merge_req[b] = b.
// Returns the number of items (B * S).
int32_t sched_plan_decode(int32_t B, const int32_t *seq_lens, int32_t S, int32_t blk,
                          int32_t *items, int32_t *merge_req, int32_t *merge_begin) {
  if (S < 1) S = 1;
  for (int32_t b = 0; b < B; ++b) {
    const int32_t len = seq_lens[b];
    int32_t chunk = (len + S - 1) / S;
    chunk = (chunk + blk - 1) / blk * blk;
    if (chunk <= 0) chunk = blk;
    for (int32_t s = 0; s < S; ++s) {
      int32_t *it = items + 4 * (b * S + s);
      int32_t begin = s * chunk;
      int32_t end = std::min(len, begin + chunk);
      if (end < begin) end = begin;
      it[0] = b;
      it[1] = begin;
      it[2] = end;
      it[3] = S == 1 ? -1 : b * S + s;
    }
    if (S > 1) {
      merge_req[b] = b;
      merge_begin[b] = b * S;
    }
  }
  if (S > 1) merge_begin[B] = B * S;
  return B * S;
}

// Per-task cost of a decode plan: tokens of the task's item (task = item * Hkv + head).
void sched_plan_task_costs(int32_t n_items, const int32_t *items, int32_t hkv, float *cost) {
  for (int32_t i = 0; i < n_items; ++i) {
    const float c = (float)(items[4 * i + 2] - items[4 * i + 1]);
    for (int32_t h = 0; h < hkv; ++h) cost[i * hkv + h] = c;
  }
}

void sched_order_grouped_lpt(const float *cost, int32_t n, int32_t block, int32_t *out) {
  grouped_lpt(cost, n, block, out);
}

// Cluster-launch-control region order: prefix [0, R) alternates heaviest and
// lightest, the suffix holds the rest heaviest first. R <= 0 or n <= R:
// grouped LPT with `block`.
void sched_order_region(const float *cost, int32_t n, int32_t R, int32_t block, int32_t *out) {
  if (R <= 0 || n <= R) {
    grouped_lpt(cost, n, block, out);
    return;
  }
  std::vector<int32_t> lpt(n);
  std::iota(lpt.begin(), lpt.end(), 0);
  std::stable_sort(lpt.begin(), lpt.end(), [&](int a, int b) { return cost[a] > cost[b]; });
  const int32_t nh = (R + 1) / 2, nl = R - nh;
  for (int32_t i = 0; i < nh; ++i) out[2 * i] = lpt[i];
  for (int32_t i = 0; i < nl; ++i) out[2 * i + 1] = lpt[n - 1 - i];
  int32_t k = R;
  for (int32_t i = nh; i < n - nl; ++i) out[k++] = lpt[i];
}

}  // extern "C"
