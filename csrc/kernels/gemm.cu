// gemm.cu -- bf16 GEMM on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
//   Y[T, N] = X[T, K] . W[N, K]^T          (Linear layer, weights row-major)
//
// Decode-first design ("swap-AB"): the MMA's M dimension runs over 128 rows
// of the weight (output features) and its N dimension over a tile of TN
// tokens (16..256). A decode step has few tokens and many weight rows, so the
// weight stream -- the HBM-bound part -- always fills the 128-row MMA, and the
// token count only sets the (cheap) N width. Prefill uses TN = 256.
//
// Persistent stream-K schedule: the k-block iterations of all tiles
// (tiles x K/64) are split into `grid` contiguous, equal ranges, one per CTA
// (at most one CTA per SM), so every SM streams the same number of weight
// bytes no matter how the tile count divides the SM count. A CTA's range
// covers one or more tile *segments*. A tile covered by one segment is
// finished in place; otherwise each segment stores its fp32 partial into a
// workspace slice of its CTA (two per CTA: only a CTA's first and last
// segments can be partial) and bumps the tile's arrival counter, and the last
// segment to arrive sums the slices in segment order (fixed order: results
// are bit-reproducible), applies the epilogue and resets the counter to zero.
//
// One CTA = 6 warps:
//   warp 0  TMA producer: streams W and X K-blocks (64 elements = one
//           128-byte swizzle atom) through an STAGES-deep ring, continuously
//           across segment boundaries;
//   warp 1  MMA issuer: 4 x tcgen05.mma (K = 16) per stage into one of two
//           TMEM accumulators [128 lanes x TN columns] (segments alternate);
//           tcgen05.commit frees each stage as its MMAs retire;
//   warps 2-5 epilogue: tcgen05.ld the finished accumulator while the MMA
//           warp already fills the other one, stage 16-token slabs in shared
//           memory, write coalesced rows.
//
// Programmatic dependent launch: the producer issues the weight loads of the
// first stages before griddepcontrol.wait (weights do not depend on the
// previous kernel), then the activation loads; the epilogue waits before its
// first global write. Every CTA triggers its dependents at entry.
//
// Epilogues: plain store; SwiGLU over an interleaved gate/up weight whose
// 128-row tile holds 64 gate rows followed by the matching 64 up rows
// (out[t, j] = silu(gate) * up); and RoPE + KV append for the fused QKV
// projection, where a 128-row tile is exactly one head: query heads are
// rotated into the attention input, key heads rotated and value heads copied
// straight into their page slots of the paged KV cache; and the fused
// all-reduce of a row-parallel projection (see publish_tile /
// reduce_owned_chunks): each finished tile is pushed over NVLink as the MMA
// warp is already working on the next one, so the transfer overlaps the math
// tile by tile.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <stdexcept>

#include "common.cuh"
#include "gemm_api.h"
#include "sched/ptx.cuh"
#include "tmap.h"

namespace gemm {

constexpr int BM = 128;  // weight rows per tile (MMA M)
constexpr int BK = 64;   // K elements per stage (128 bytes of bf16)
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;
constexpr int kSlab = 16;  // tokens per epilogue slab
constexpr int kSlabPitch = BM + 4;

template <int TN>
struct Cfg {
  static constexpr int W_BYTES = BM * BK * 2;
  static constexpr int X_BYTES = TN * BK * 2;
  static constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 12 ? 12 : (200 * 1024) / STAGE_BYTES;
  static constexpr int ACC_COLS = TN < 32 ? 32 : TN;  // one accumulator
  static constexpr int TMEM_COLS = 2 * ACC_COLS;       // two accumulators
  static constexpr int SLAB_BYTES = kSlab * kSlabPitch * 4;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + SLAB_BYTES + 512;
  static constexpr int smem(int stages) { return 1024 + stages * STAGE_BYTES + SLAB_BYTES + 512; }
  // cluster split-K: each CTA's fp32 partial tile [TN][128] lives in shared
  // memory for its peers to read over DSMEM
  static constexpr int RED_BYTES = TN * BM * 4;
  static constexpr int CSTAGES_RAW = (200 * 1024 - RED_BYTES) / STAGE_BYTES;
  static constexpr int CSTAGES = CSTAGES_RAW > 12 ? 12 : CSTAGES_RAW;
  static constexpr int CSMEM = 1024 + CSTAGES * STAGE_BYTES + SLAB_BYTES + RED_BYTES + 512;
};

struct Params {
  GemmArgs a;
  int n_tiles, t_tiles, kb, tiles;
  long long units;  // tiles * kb
  int grid;
  int stages;  // ring depth of this launch (<= Cfg<TN>::STAGES)
  int cs;      // cluster split-K: CTAs per cluster (0: stream-K kernel)
  int pw = 0, ps = 1;  // pair kernel: tiles [0, pw) whole, the rest in ps k-ranges each (ps <= 1: none)
};

// Residual add + RMSNorm of the output rows a CTA completes (defined below;
// out of line, and only called when the launch fuses the norm).
// Only scalars cross this call: taking the address of the kernel's Params
// (a reference argument) would make the compiler copy them to local memory
// for the whole kernel.
__device__ __noinline__ void finish_rows_impl(const __nv_bfloat16 *y, int ldy, int N, __nv_bfloat16 *res,
                                              const __nv_bfloat16 *w, __nv_bfloat16 *out, uint32_t *cnt, float eps,
                                              int n_tiles, int r0, int nrows, int et, float *scratch);
__device__ __forceinline__ void finish_rows(const Params &p, int r0, int nrows, int et, float *scratch) {
  const GemmArgs &a = p.a;
  if (a.norm_w != nullptr && nrows > 0)
    finish_rows_impl(static_cast<const __nv_bfloat16 *>(a.y), a.ldy, a.N, a.norm_res, a.norm_w, a.norm_out,
                     a.row_cnt, a.norm_eps, p.n_tiles, r0, nrows, et, scratch);
}

// One segment: the k-block range [kb0, kb1) of `tile` handled by one CTA.
struct Seg {
  int tile, kb0, kb1;
  int seg, nsegs;  // position among the tile's segments
};

__device__ __forceinline__ long long cta_begin(const Params &p, int c) {
  return (long long)c * p.units / p.grid;
}
__device__ __forceinline__ int cta_of_unit(const Params &p, long long u) {
  return (int)(((u + 1) * p.grid - 1) / p.units);
}

// The k-th segment of CTA c; false when c has fewer segments. Every role
// derives the same sequence from the CTA index, so no hand-off is needed.
__device__ __forceinline__ bool segment(const Params &p, int c, int k, Seg &s) {
  const long long b = cta_begin(p, c), e = cta_begin(p, c + 1);
  if (b >= e) return false;
  const int tile = (int)(b / p.kb) + k;
  const long long tb = (long long)tile * p.kb, te = tb + p.kb;
  if (tb >= e) return false;
  const long long lo = max(b, tb), hi = min(e, te);
  s.tile = tile;
  s.kb0 = (int)(lo - tb);
  s.kb1 = (int)(hi - tb);
  const int c0 = cta_of_unit(p, tb), c1 = cta_of_unit(p, te - 1);
  s.seg = c - c0;
  s.nsegs = c1 - c0 + 1;
  return true;
}

// Epilogue writer: token row v[0..127] (fp32, shared memory) of tile
// (n_tile, token t); thread k of 8 writes its share.
// A low-latency all-reduce line: 8 bytes of payload (two bf16x2 words) and
// the call's epoch beside each, in one 16-byte store. Each 8-byte half lands
// whole, so a reader that sees the epoch in a half has that half's payload.
__device__ __forceinline__ void st_ll(uint4 *dst, uint32_t d0, uint32_t d1, uint32_t e) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(d0), "r"(e), "r"(d1), "r"(e)
               : "memory");
}

// The same line through the multicast mapping: two 8-byte integer multimem
// stores, one per half {payload, epoch}; the switch writes every rank's copy.
__device__ __forceinline__ void st_ll_mc(uint4 *dst, uint32_t d0, uint32_t d1, uint32_t e) {
  const uint64_t h0 = ((uint64_t)e << 32) | d0, h1 = ((uint64_t)e << 32) | d1;
  asm volatile("multimem.st.relaxed.sys.global.b64 [%0], %1;" ::"l"(dst), "l"(h0) : "memory");
  asm volatile("multimem.st.relaxed.sys.global.b64 [%0], %1;" ::"l"(reinterpret_cast<uint8_t *>(dst) + 8), "l"(h1)
               : "memory");
}

template <int EPI>
__device__ __forceinline__ void write_row(const GemmArgs &a, int n_tile, int t, const float *v,
                                          int k, uint32_t ll_e = 0) {
  if (EPI == kEpiStore) {
    const int c = k * 16;
    uint4 o0, o1;
    o0.x = pack_bf16x2(v[c + 0], v[c + 1]);
    o0.y = pack_bf16x2(v[c + 2], v[c + 3]);
    o0.z = pack_bf16x2(v[c + 4], v[c + 5]);
    o0.w = pack_bf16x2(v[c + 6], v[c + 7]);
    o1.x = pack_bf16x2(v[c + 8], v[c + 9]);
    o1.y = pack_bf16x2(v[c + 10], v[c + 11]);
    o1.z = pack_bf16x2(v[c + 12], v[c + 13]);
    o1.w = pack_bf16x2(v[c + 14], v[c + 15]);
    uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(a.y) +
                                           (size_t)t * a.ldy + n_tile * BM + c);
    dst[0] = o0;
    dst[1] = o1;
  } else if (EPI == kEpiSwiGLU) {
    const int c = k * 8;  // 8 gate rows; their up rows sit 64 rows further
    float g[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] = silu(v[c + j]) * v[c + 64 + j];
    uint4 o;
    o.x = pack_bf16x2(g[0], g[1]);
    o.y = pack_bf16x2(g[2], g[3]);
    o.z = pack_bf16x2(g[4], g[5]);
    o.w = pack_bf16x2(g[6], g[7]);
    *reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(a.y) + (size_t)t * a.ldy +
                               n_tile * (BM / 2) + c) = o;
  } else if (EPI == kEpiAllReduce || EPI == kEpiReduceScatter) {
    const int c = k * 16;
    uint4 o0, o1;
    o0.x = pack_bf16x2(v[c + 0], v[c + 1]);
    o0.y = pack_bf16x2(v[c + 2], v[c + 3]);
    o0.z = pack_bf16x2(v[c + 4], v[c + 5]);
    o0.w = pack_bf16x2(v[c + 6], v[c + 7]);
    o1.x = pack_bf16x2(v[c + 8], v[c + 9]);
    o1.y = pack_bf16x2(v[c + 10], v[c + 11]);
    o1.z = pack_bf16x2(v[c + 12], v[c + 13]);
    o1.w = pack_bf16x2(v[c + 14], v[c + 15]);
    const size_t off = ((size_t)a.rank * a.T + t) * a.N + (size_t)n_tile * BM + c;
    if (EPI == kEpiAllReduce && a.ll_state != nullptr) {
      // low-latency lines into every rank's buffer (set of this call's epoch)
      const size_t line = (size_t)(ll_e & 1u) * a.ll_set_lines + off / 4;
      if (a.ll_mc != nullptr) {
        uint4 *dst = reinterpret_cast<uint4 *>(a.ll_mc) + line;
        st_ll_mc(dst, o0.x, o0.y, ll_e);
        st_ll_mc(dst + 1, o0.z, o0.w, ll_e);
        st_ll_mc(dst + 2, o1.x, o1.y, ll_e);
        st_ll_mc(dst + 3, o1.z, o1.w, ll_e);
      } else {
        for (int j = 0; j < a.world; ++j) {
          uint4 *dst = reinterpret_cast<uint4 *>(a.recv[j]) + line;
          st_ll(dst, o0.x, o0.y, ll_e);
          st_ll(dst + 1, o0.z, o0.w, ll_e);
          st_ll(dst + 2, o1.x, o1.y, ll_e);
          st_ll(dst + 3, o1.z, o1.w, ll_e);
        }
      }
    } else if (EPI == kEpiAllReduce) {
      for (int j = 0; j < a.world; ++j) {  // NVLink stores into every rank's slab
        uint4 *dst = reinterpret_cast<uint4 *>(a.recv[j] + off);
        dst[0] = o0;
        dst[1] = o1;
      }
    } else {  // only the owner of the token reduces it
      uint4 *dst = reinterpret_cast<uint4 *>(a.recv[sp_row_owner(t, a.T, a.world)] + off);
      dst[0] = o0;
      dst[1] = o1;
    }
  } else {  // kEpiRopeKV: the tile is one head
    const int h = n_tile;
    const int c = k * 8;  // rotate pairs (c + j, c + j + 64)
    __nv_bfloat16 *dst;
    bool rotate = true;
    if (h < a.Hq) {
      dst = a.q_out + ((size_t)t * a.Hq + h) * BM;
    } else {
      const int s = a.slot[t];
      if (s < 0) return;  // padding row: no cache write
      if (a.kv_pages > 0 && (long long)s >= (long long)a.kv_pages * a.page_size) {
        report_bad_index(a.status, kSiteKvSlot, s);
        return;
      }
      const int page = s / a.page_size, off = s % a.page_size;
      const bool is_k = h < a.Hq + a.Hkv;
      const int kvh = is_k ? h - a.Hq : h - a.Hq - a.Hkv;
      __nv_bfloat16 *cache = is_k ? a.k_cache : a.v_cache;
      dst = cache + (((size_t)page * a.Hkv + kvh) * a.page_size + off) * BM;
      rotate = is_k;
    }
    float lo[8], hi[8];
    if (rotate) {
      const float2 *cs = reinterpret_cast<const float2 *>(a.cos_sin) + (size_t)a.pos[t] * (BM / 2) + c;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float2 r = cs[j];
        const float x = v[c + j], y = v[c + 64 + j];
        lo[j] = x * r.x - y * r.y;
        hi[j] = y * r.x + x * r.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        lo[j] = v[c + j];
        hi[j] = v[c + 64 + j];
      }
    }
    uint4 o;
    o.x = pack_bf16x2(lo[0], lo[1]);
    o.y = pack_bf16x2(lo[2], lo[3]);
    o.z = pack_bf16x2(lo[4], lo[5]);
    o.w = pack_bf16x2(lo[6], lo[7]);
    *reinterpret_cast<uint4 *>(dst + c) = o;
    o.x = pack_bf16x2(hi[0], hi[1]);
    o.y = pack_bf16x2(hi[2], hi[3]);
    o.z = pack_bf16x2(hi[4], hi[5]);
    o.w = pack_bf16x2(hi[6], hi[7]);
    *reinterpret_cast<uint4 *>(dst + 64 + c) = o;
  }
}

// All-reduce, part 1: after this rank's partial of `tile` has been stored
// into every rank's slab, raise the flag of each 16-token chunk of the tile
// on every rank (release at system scope: the data is visible to the reader
// that acquires the flag). Flag (src, tile, chunk) lives in the reader's array.
template <int TN>
__device__ __forceinline__ void publish_tile(const Params &p, int tile, int et) {
  const GemmArgs &a = p.a;
  constexpr int CH = TN / kSlab;
  __threadfence_system();
  named_bar(1, kEpiThreads);
  const int tt = tile % p.t_tiles;
  const int chunks = (min(TN, a.T - tt * TN) + kSlab - 1) / kSlab;
  for (int i = et; i < a.world * chunks; i += kEpiThreads) {
    const int j = i / chunks, ch = i % chunks;
    ptx::st_release_sys(a.flags[j] + ((size_t)a.rank * p.tiles + tile) * CH + ch, 1u);
  }
}

// How many flag releases chunk `ch` of token tile `tt` receives from one rank:
// 1 under stream-K (one CTA writes the whole tile); under cluster split-K each
// cluster rank releases the chunks its share of tokens [r*tv/cs, (r+1)*tv/cs)
// touches, so the count is the number of shares that intersect the chunk.
template <int TN>
__device__ __forceinline__ uint32_t chunk_contributors(const Params &p, int tt, int ch) {
  if (p.cs <= 1) return 1u;
  const int tv = min(TN, p.a.T - tt * TN);
  const int c0 = ch * kSlab, c1 = min(c0 + kSlab, tv);
  uint32_t n = 0;
  for (int r = 0; r < p.cs; ++r) {
    const int lo = r * tv / p.cs, hi = (r + 1) * tv / p.cs;
    n += (lo < hi && lo < c1 && hi > c0) ? 1u : 0u;
  }
  return n;
}

// Cluster split-K, all-reduce epilogue: after this CTA pushed its token rows
// [lo, hi) of a tile to every rank, release each chunk those rows touch
// (one count per chunk and rank; readers wait for chunk_contributors).
template <int TN>
__device__ __forceinline__ void publish_rows(const Params &p, int tile, int lo, int hi, int et) {
  const GemmArgs &a = p.a;
  constexpr int CH = TN / kSlab;
  __threadfence_system();
  named_bar(1, kEpiThreads);
  if (lo >= hi) return;
  const int c_first = lo / kSlab, c_last = (hi - 1) / kSlab;
  const int chunks = c_last - c_first + 1;
  for (int i = et; i < a.world * chunks; i += kEpiThreads) {
    const int j = i / chunks, ch = c_first + i % chunks;
    ptx::red_add_release_sys(a.flags[j] + ((size_t)a.rank * p.tiles + tile) * CH + ch, 1u);
  }
}

// Reduce-scatter: after this CTA stored the token rows [lo, hi) of `tile`
// (tile-local row indices) into their owners' slabs, raise each row's flag
// (source = this rank, n-tile, token) in the owner's row-flag array. Every
// row is written by exactly one CTA (stream-K: the tile's finishing segment;
// cluster split-K: the cluster rank whose share holds it), so the owner waits
// for the value 1.
template <int TN>
__device__ __forceinline__ void publish_rows_rs(const Params &p, int tile, int lo, int hi, int et) {
  const GemmArgs &a = p.a;
  __threadfence_system();
  named_bar(1, kEpiThreads);
  const int nt = tile / p.t_tiles, t0 = (tile % p.t_tiles) * TN;
  for (int r = lo + et; r < hi; r += kEpiThreads) {
    const int t = t0 + r;
    uint32_t *f = a.flags[sp_row_owner(t, a.T, a.world)] + ((size_t)a.rank * p.n_tiles + nt) * a.T + t;
    ptx::st_release_sys(f, 1u);
  }
}

__device__ __forceinline__ uint4 ld_volatile_v4(const uint32_t *p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Gathered activations: the producer lane waits until the rows [r0, r1) of X
// have been raised in x_ready (r0 is a multiple of 16). Flags are polled
// eight 16-byte vectors at a time (the loads of a batch are in flight
// together); once all are set, a system-scope fence turns the observation
// into an acquire of the owners' releases, and a proxy fence orders it
// before this thread's TMA (async-proxy) reads of the rows. On timeout the
// status word is set and the loads go ahead (no hang). The budget is half of
// the MMA warp's wait on the stage, so a missing row ends as a peer timeout
// and the stage still lands before the MMA warp gives up on it.
__device__ __noinline__ void wait_rows_ready(const uint32_t *ready, int r0, int r1, int *status) {
  constexpr uint64_t kReadyBudgetNs = kWaitBudgetNs / 2;
  const uint64_t start = ptx::globaltimer_ns();
  for (;;) {
    bool all = true;
    for (int t = r0; t < r1; t += 32) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (t + 4 * u < r1) v[u] = ld_volatile_v4(ready + t + 4 * u);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int b = t + 4 * u;
        if (b < r1)
          all = all && v[u].x != 0u && (b + 1 >= r1 || v[u].y != 0u) && (b + 2 >= r1 || v[u].z != 0u) &&
                (b + 3 >= r1 || v[u].w != 0u);
      }
    }
    if (all) break;
    if (ptx::globaltimer_ns() - start > kReadyBudgetNs) {
      report_status(status, kStatusPeerTimeout);
      return;
    }
  }
  ptx::fence_acq_rel_sys();
  ptx::fence_proxy_async_global();
}

// All-reduce, part 2: the reduction units are (tile, 16-token chunk); CTA c
// owns units c, c + grid, ... on every rank (the same assignment everywhere,
// independent of timing). For each owned unit it waits for the chunk flags
// of all ranks, sums their partials in rank order (the same order on every
// rank: bit-identical results), writes the bf16 output and clears its flags.
// Pushes never wait, so no wait can form a cycle.
template <int TN>
__device__ void reduce_owned_chunks(const Params &p, int c, int et, float *scratch) {
  const GemmArgs &a = p.a;
  constexpr int CH = TN / kSlab;
  const __nv_bfloat16 *mine = a.recv[a.rank];
  uint32_t *my_flags = a.flags[a.rank];
  const int units = p.tiles * CH;
  for (int u = c; u < units; u += p.grid) {
    const int tile = u / CH, ch = u % CH;
    const int nt = tile / p.t_tiles, tt = tile % p.t_tiles;
    const int t0 = tt * TN + ch * kSlab;
    if (t0 >= a.T) continue;  // uniform across the CTA
    const int tmax = min(kSlab, a.T - t0);
    if (et < a.world) {
      const uint32_t *f = my_flags + ((size_t)et * p.tiles + tile) * CH + ch;
      const uint32_t need = chunk_contributors<TN>(p, tt, ch);
      bool ok = ptx::ld_acquire_sys(f) >= need;
      if (!ok) {
        const uint64_t start = ptx::globaltimer_ns();
        while (!ok) {
          for (int i = 0; i < 64 && !ok; ++i) ok = ptx::ld_acquire_sys(f) >= need;
          if (!ok && ptx::globaltimer_ns() - start > kWaitBudgetNs) break;
        }
        if (!ok) report_status(a.status, kStatusPeerTimeout);
      }
    }
    named_bar(1, kEpiThreads);
    // 16 tokens x 128 columns: thread et handles token et / 8, 16 columns
    const int tl = et / 8, col = (et % 8) * 16;
    if (tl < tmax) {
      const int t = t0 + tl;
      float acc[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[j] = 0.f;
      for (int src = 0; src < a.world; ++src) {
        const uint4 *q = reinterpret_cast<const uint4 *>(
            mine + ((size_t)src * a.T + t) * a.N + (size_t)nt * BM + col);
        const uint4 u0 = __ldcv(q), u1 = __ldcv(q + 1);
        const __nv_bfloat16 *e0 = reinterpret_cast<const __nv_bfloat16 *>(&u0);
        const __nv_bfloat16 *e1 = reinterpret_cast<const __nv_bfloat16 *>(&u1);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc[j] += __bfloat162float(e0[j]);
          acc[8 + j] += __bfloat162float(e1[j]);
        }
      }
      uint4 o0, o1;
      o0.x = pack_bf16x2(acc[0], acc[1]);
      o0.y = pack_bf16x2(acc[2], acc[3]);
      o0.z = pack_bf16x2(acc[4], acc[5]);
      o0.w = pack_bf16x2(acc[6], acc[7]);
      o1.x = pack_bf16x2(acc[8], acc[9]);
      o1.y = pack_bf16x2(acc[10], acc[11]);
      o1.z = pack_bf16x2(acc[12], acc[13]);
      o1.w = pack_bf16x2(acc[14], acc[15]);
      uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(a.y) + (size_t)t * a.ldy +
                                             (size_t)nt * BM + col);
      dst[0] = o0;
      dst[1] = o1;
    }
    named_bar(1, kEpiThreads);
    if (et < a.world) my_flags[((size_t)et * p.tiles + tile) * CH + ch] = 0u;
    finish_rows(p, t0, tmax, et, scratch);
  }
}

// ---------------------------------------------------------------------------
// Residual add + RMSNorm fused after the projection (GemmArgs::norm_w).
//
// One output row, normalised by the 128 epilogue threads with the arithmetic
// of sched_add_rmsnorm's NTV-thread kernel (elementwise.cu): NTV virtual
// threads, virtual thread vt = et + 128 m owning the 8-element vectors
// (vt + i NTV) * 8, i < 2; per-thread sums in the same order, the same xor
// shuffle tree per virtual warp (virtual warp et / 32 + 4 m has the lanes of
// real warp et / 32) and the virtual warps' sums added in index order, so
// the results are bit-identical to the separate kernel.
template <int NTV>
__device__ __forceinline__ void norm_row(const __nv_bfloat16 *y, int ldy, int H, __nv_bfloat16 *res_base,
                                         const __nv_bfloat16 *nw, __nv_bfloat16 *out, float eps, int t, int et,
                                         float *red) {
  constexpr int M = NTV / 128;
  const int lane = et & 31, rw = et >> 5;
  const __nv_bfloat16 *x = y + (size_t)t * ldy;
  __nv_bfloat16 *res = res_base + (size_t)t * H;
  // pass 1: res += x (rounded to bf16 once) and the per-virtual-thread sums
#pragma unroll
  for (int m = 0; m < M; ++m) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int c = (et + 128 * m + i * NTV) * 8;
      if (c < H) {
        const uint4 xv = __ldcg(reinterpret_cast<const uint4 *>(x + c));  // rows other CTAs wrote
        const uint4 rv = *reinterpret_cast<const uint4 *>(res + c);
        const __nv_bfloat16 *xe = reinterpret_cast<const __nv_bfloat16 *>(&xv);
        const __nv_bfloat16 *re = reinterpret_cast<const __nv_bfloat16 *>(&rv);
        uint4 ov;
        __nv_bfloat16 *oe = reinterpret_cast<__nv_bfloat16 *>(&ov);
#pragma unroll
        for (int j = 0; j < 8; ++j) oe[j] = __float2bfloat16(__bfloat162float(xe[j]) + __bfloat162float(re[j]));
        *reinterpret_cast<uint4 *>(res + c) = ov;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float v = __bfloat162float(oe[j]);
          ss += v * v;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[rw + 4 * m] = ss;
  }
  named_bar(1, kEpiThreads);
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < NTV / 32; ++i) tot += red[i];
  const float inv = rsqrtf(tot / (float)H + eps);
  // pass 2: the values are the bf16 sums this thread just stored, read back
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int c = (et + 128 * m + i * NTV) * 8;
      if (c < H) {
        const uint4 rv = *reinterpret_cast<const uint4 *>(res + c);
        const uint4 wv = *reinterpret_cast<const uint4 *>(nw + c);
        const __nv_bfloat16 *re = reinterpret_cast<const __nv_bfloat16 *>(&rv);
        const __nv_bfloat16 *we = reinterpret_cast<const __nv_bfloat16 *>(&wv);
        float vv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) vv[j] = __bfloat162float(re[j]);
        uint4 ov;
        ov.x = pack_bf16x2(vv[0] * inv * __bfloat162float(we[0]), vv[1] * inv * __bfloat162float(we[1]));
        ov.y = pack_bf16x2(vv[2] * inv * __bfloat162float(we[2]), vv[3] * inv * __bfloat162float(we[3]));
        ov.z = pack_bf16x2(vv[4] * inv * __bfloat162float(we[4]), vv[5] * inv * __bfloat162float(we[5]));
        ov.w = pack_bf16x2(vv[6] * inv * __bfloat162float(we[6]), vv[7] * inv * __bfloat162float(we[7]));
        *reinterpret_cast<uint4 *>(out + (size_t)t * H + c) = ov;
      }
    }
  named_bar(1, kEpiThreads);  // red is rewritten by the next row
}

// Called by all 128 epilogue threads after they wrote output rows
// [r0, r0 + nrows) of n-tile nt: counts the n-tile against each row and
// normalises the rows this CTA completed. `scratch` is shared memory of at
// least (nrows + 4 + 32) words that no other role uses meanwhile.
__device__ __noinline__ void finish_rows_impl(const __nv_bfloat16 *y, int ldy, int N, __nv_bfloat16 *res,
                                              const __nv_bfloat16 *w, __nv_bfloat16 *out, uint32_t *cnt, float eps,
                                              int n_tiles, int r0, int nrows, int et, float *scratch) {
  int *fin = reinterpret_cast<int *>(scratch);
  int *nfin = fin + nrows;
  float *red = scratch + nrows + 4;
  __threadfence();  // this thread's row stores are visible before its count
  if (et == 0) *nfin = 0;
  named_bar(1, kEpiThreads);
  for (int r = et; r < nrows; r += kEpiThreads) {
    const int t = r0 + r;
    if (atomicAdd(cnt + t, 1u) == (uint32_t)(n_tiles - 1)) {
      cnt[t] = 0u;  // zero for the next call
      fin[atomicAdd(nfin, 1)] = t;
    }
  }
  __threadfence();  // the other CTAs' stores of the rows we complete are visible to our reads
  named_bar(1, kEpiThreads);
  const int nf = *nfin;
  for (int i = 0; i < nf; ++i) {
    const int t = fin[i];
    if (N <= 4096)
      norm_row<256>(y, ldy, N, res, w, out, eps, t, et, red);
    else if (N <= 8192)
      norm_row<512>(y, ldy, N, res, w, out, eps, t, et, red);
    else
      norm_row<1024>(y, ldy, N, res, w, out, eps, t, et, red);
  }
  named_bar(1, kEpiThreads);  // scratch reuse by the caller
}

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// The epoch of this call (low-latency exchange): every CTA reads the same
// value, since only the call's last CTA advances it (ll_finish).
__device__ __forceinline__ uint32_t ll_epoch(const GemmArgs &a) {
  return a.ll_state != nullptr ? ld_volatile_u32(a.ll_state) + 1u : 0u;
}

// Called by one thread of every CTA after its last read of the line buffer:
// the last CTA of the launch resets the counter and advances the epoch
// (skipping 0 on wrap-around, so a never-written line never matches).
__device__ __forceinline__ void ll_finish(const GemmArgs &a) {
  __threadfence();
  if (atomicAdd(a.ll_state + 1, 1u) == gridDim.x - 1) {
    a.ll_state[1] = 0u;
    const uint32_t e = ld_volatile_u32(a.ll_state) + 1u;
    __threadfence();
    a.ll_state[0] = e == 0xFFFFFFFFu ? 1u : e;
  }
}

// One thread's share of a reduced row in the low-latency exchange: load the
// four lines of EVERY source in one round of independent loads, re-poll only
// the sources whose halves do not yet carry the call's epoch (bounded), then
// sum in rank order (fp32) and store 16 output columns. (Polling the sources
// one after another put world dependent load round trips on every call.)
__device__ __forceinline__ void reduce_line_row(const GemmArgs &a, const uint4 *mine, int nt, int t, int col,
                                                uint32_t e) {
  uint2 pl[kMaxWorld][4];  // payload words of each source's four lines, once they carry the epoch
  const uint4 *base = mine + (((size_t)t * a.N + (size_t)nt * BM + col) / 4);
  const size_t src_stride = (size_t)a.T * a.N / 4;  // lines between sources
  uint32_t pending = a.world >= 32 ? 0xFFFFFFFFu : ((1u << a.world) - 1u);
  uint64_t start = 0;
  for (uint32_t polls = 0; pending != 0u; ++polls) {
#pragma unroll
    for (int src = 0; src < kMaxWorld; ++src) {
      if (!(pending & (1u << src))) continue;
      const uint4 *q = base + (size_t)src * src_stride;
      uint4 l[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) l[i] = ld_volatile_v4(reinterpret_cast<const uint32_t *>(q + i));
      bool ok = true;
#pragma unroll
      for (int i = 0; i < 4; ++i) ok = ok && l[i].y == e && l[i].w == e;
      if (ok) {
#pragma unroll
        for (int i = 0; i < 4; ++i) pl[src][i] = make_uint2(l[i].x, l[i].z);
        pending &= ~(1u << src);
      }
    }
    if (pending != 0u && (polls & 63u) == 0u) {
      const uint64_t now = ptx::globaltimer_ns();
      if (start == 0) {
        start = now;
      } else if (now - start > kWaitBudgetNs) {
        report_status(a.status, kStatusPeerTimeout);
#pragma unroll
        for (int src = 0; src < kMaxWorld; ++src)
          if (pending & (1u << src))
#pragma unroll
            for (int i = 0; i < 4; ++i) pl[src][i] = make_uint2(0u, 0u);
        break;
      }
    }
  }
  float acc[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j] = 0.f;
#pragma unroll
  for (int src = 0; src < kMaxWorld; ++src) {  // rank order: the same sums as the flag path
    if (src >= a.world) break;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat16 *lo = reinterpret_cast<const __nv_bfloat16 *>(&pl[src][i].x);
      const __nv_bfloat16 *hi = reinterpret_cast<const __nv_bfloat16 *>(&pl[src][i].y);
      acc[4 * i] += __bfloat162float(lo[0]);
      acc[4 * i + 1] += __bfloat162float(lo[1]);
      acc[4 * i + 2] += __bfloat162float(hi[0]);
      acc[4 * i + 3] += __bfloat162float(hi[1]);
    }
  }
  uint4 o0, o1;
  o0.x = pack_bf16x2(acc[0], acc[1]);
  o0.y = pack_bf16x2(acc[2], acc[3]);
  o0.z = pack_bf16x2(acc[4], acc[5]);
  o0.w = pack_bf16x2(acc[6], acc[7]);
  o1.x = pack_bf16x2(acc[8], acc[9]);
  o1.y = pack_bf16x2(acc[10], acc[11]);
  o1.z = pack_bf16x2(acc[12], acc[13]);
  o1.w = pack_bf16x2(acc[14], acc[15]);
  uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(a.y) + (size_t)t * a.ldy +
                                         (size_t)nt * BM + col);
  dst[0] = o0;
  dst[1] = o1;
}

// All-reduce, part 2 of the low-latency exchange: the same owned units and
// rank-order sums as reduce_owned_chunks, but each thread polls its own four
// lines per source until they carry the call's epoch (bounded), with no
// flags or fences; the rows of a unit are then counted for the fused norm.
template <int TN>
__device__ void reduce_owned_chunks_ll(const Params &p, int c, int et, uint32_t e, float *scratch) {
  const GemmArgs &a = p.a;
  constexpr int CH = TN / kSlab;
  const uint4 *mine = reinterpret_cast<const uint4 *>(a.recv[a.rank]) + (size_t)(e & 1u) * a.ll_set_lines;
  const int units = p.tiles * CH;
  const int tl = et / 8, col = (et % 8) * 16;
  for (int u = c; u < units; u += p.grid) {
    const int tile = u / CH, ch = u % CH;
    const int nt = tile / p.t_tiles, tt = tile % p.t_tiles;
    const int t0 = tt * TN + ch * kSlab;
    if (t0 >= a.T) continue;  // uniform across the CTA
    const int tmax = min(kSlab, a.T - t0);
    if (tl < tmax) reduce_line_row(a, mine, nt, t0 + tl, col, e);
    finish_rows(p, t0, tmax, et, scratch);
  }
}

template <int TN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                const Params p) {
  using C = Cfg<TN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *stage_mem = base;
  const int S = p.stages;
  float *slab = reinterpret_cast<float *>(base + S * C::STAGE_BYTES);
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + S * C::STAGE_BYTES + C::SLAB_BYTES);
  uint64_t *full = bars;
  uint64_t *empty = bars + S;
  uint64_t *acc_full = bars + 2 * S;       // [2]
  uint64_t *acc_empty = bars + 2 * S + 2;  // [2]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * S + 4);
  volatile int *last_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int c = blockIdx.x;
  const GemmArgs &a = p.a;

  ptx::pdl_launch_dependents();
  if (a.trace && threadIdx.x == 0) a.trace[c * 4] = ptx::globaltimer_ns();
  if (warp == 0) {
    ptx::tmem_alloc(tmem_slot, C::TMEM_COLS);
    ptx::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&acc_full[i], 1);
      ptx::mbar_init(&acc_empty[i], kEpiThreads);
    }
    ptx::fence_mbar_init();
  }
  if (threadIdx.x == 64) {
    ptx::prefetch_tmap(&tmW);
    ptx::prefetch_tmap(&tmX);
  }
  ptx::tc_fence_before();
  __syncwarp();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ============================================================ producer
    if (ptx::elect_one()) {
      // Weights of the first stages do not depend on the previous kernel:
      // fetch them before waiting for it.
      int pre = 0;
      {
        Seg s;
        for (int k = 0; pre < S && segment(p, c, k, s); ++k) {
          const int nt = s.tile / p.t_tiles;
          for (int kb = s.kb0; kb < s.kb1 && pre < S; ++kb, ++pre) {
            ptx::mbar_arrive_expect_tx(&full[pre], C::STAGE_BYTES);
            ptx::tma_load_2d(stage_mem + pre * C::STAGE_BYTES, &tmW, &full[pre], kb * BK, nt * BM);
          }
        }
      }
      ptx::pdl_wait();
      Seg s;
      int i = 0;
      bool ok = true;
      for (int k = 0; ok && segment(p, c, k, s); ++k) {
        const int nt = s.tile / p.t_tiles, tt = s.tile % p.t_tiles;
        if (a.x_ready) wait_rows_ready(a.x_ready, tt * TN, min(a.T, tt * TN + TN), a.status);
        for (int kb = s.kb0; kb < s.kb1; ++kb, ++i) {
          const int st = i % S;
          uint8_t *sm = stage_mem + st * C::STAGE_BYTES;
          if (i >= pre) {
            if (!ptx::mbar_wait(&empty[st], ((i / S) & 1) ^ 1, kWaitBudgetNs)) {
              report_status(a.status, kStatusMmaTimeout);
              ok = false;
              break;
            }
            ptx::mbar_arrive_expect_tx(&full[st], C::STAGE_BYTES);
            ptx::tma_load_2d(sm, &tmW, &full[st], kb * BK, nt * BM);
          }
          ptx::tma_load_2d(sm + C::W_BYTES, &tmX, &full[st], kb * BK, tt * TN);
        }
      }
    }
  } else if (warp == 1) {
    // ============================================================ MMA
    if (ptx::elect_one()) {
      constexpr uint32_t idesc = ptx::idesc_f16(BM, TN, /*bf16*/ 1, false, false);
      Seg s;
      int i = 0;
      bool ok = true;
      for (int k = 0; ok && segment(p, c, k, s); ++k) {
        const int ab = k & 1;
        if (!ptx::mbar_wait(&acc_empty[ab], ((k >> 1) & 1) ^ 1, kWaitBudgetNs)) {
          report_status(a.status, kStatusEpilogueTimeout);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t acc = tmem + ab * C::ACC_COLS;
        for (int kb = s.kb0; kb < s.kb1; ++kb, ++i) {
          const int st = i % S;
          if (!ptx::mbar_wait(&full[st], (i / S) & 1, kWaitBudgetNs)) {
            report_status(a.status, kStatusTmaTimeout);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          uint8_t *sm = stage_mem + st * C::STAGE_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t da = ptx::smem_desc(sm + kk * 32, 16, 1024, ptx::kLayoutSW128);
            const uint64_t db = ptx::smem_desc(sm + C::W_BYTES + kk * 32, 16, 1024, ptx::kLayoutSW128);
            ptx::mma_f16_ss(acc, da, db, idesc, (kb > s.kb0 || kk > 0) ? 1u : 0u);
          }
          ptx::mma_commit(&empty[st]);
        }
        ptx::mma_commit(&acc_full[ab]);  // fires when the segment's MMAs retire
      }
    }
  } else {
    // ============================================================ epilogue
    const int et = threadIdx.x - 64;       // 0..127
    const int q = warp & 3;                // TMEM lane quarter of this warp
    const int row = q * 32 + lane;         // accumulator row = weight row in the tile
    const int tj = et / 8, part = et % 8;  // slab token / writer share
    ptx::pdl_wait();
    const uint32_t ll_e = EPI == kEpiAllReduce ? ll_epoch(a) : 0u;  // low-latency exchange: this call's epoch
    const bool ll = EPI == kEpiAllReduce && a.ll_state != nullptr;
    Seg s;
    for (int k = 0; segment(p, c, k, s); ++k) {
      const int ab = k & 1;
      const bool waited = ptx::mbar_wait(&acc_full[ab], (k >> 1) & 1, kWaitBudgetNs);
      if (!waited) report_status(a.status, kStatusEpilogueTimeout);
      ptx::tc_fence_after();
      const int nt = s.tile / p.t_tiles, tt = s.tile % p.t_tiles;
      const int t0 = tt * TN;
      const bool direct = s.nsegs == 1;
      // two partial slots per CTA: slot 1 for the segment that opens its tile
      // (the CTA's last segment), slot 0 for a continuation (its first)
      float *wsl = direct ? nullptr : a.ws + ((size_t)c * 2 + (s.seg == 0 ? 1 : 0)) * ((size_t)TN * BM);
      for (int ch = 0; ch < TN / kSlab; ++ch) {
        if (t0 + ch * kSlab >= a.T) break;
        uint32_t r[16];
        ptx::tmem_ld16(tmem + ab * C::ACC_COLS + ((uint32_t)(q * 32) << 16) + ch * kSlab, r);
        ptx::tmem_ld_wait();
        if (!waited) {
#pragma unroll
          for (int j = 0; j < 16; ++j) r[j] = 0u;
        }
        if (direct) {
#pragma unroll
          for (int j = 0; j < 16; ++j) slab[j * kSlabPitch + row] = __uint_as_float(r[j]);
          named_bar(1, kEpiThreads);
          const int t = t0 + ch * kSlab + tj;
          if (t < a.T) write_row<EPI>(a, nt, t, slab + tj * kSlabPitch, part, ll_e);
          named_bar(1, kEpiThreads);
        } else {
          // partial slice [TN tokens][128 rows]: a warp stores 32 consecutive rows
#pragma unroll
          for (int j = 0; j < 16; ++j)
            __stcg(wsl + (size_t)(ch * kSlab + j) * BM + row, __uint_as_float(r[j]));
        }
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(&acc_empty[ab]);  // the MMA warp may refill this accumulator
      if (EPI == kEpiAllReduce && direct && !ll) publish_tile<TN>(p, s.tile, et);
      if (EPI == kEpiReduceScatter && direct) publish_rows_rs<TN>(p, s.tile, 0, min(TN, a.T - t0), et);
      if (EPI == kEpiStore && direct) finish_rows(p, t0, min(TN, a.T - t0), et, slab);
      if (!direct) {
        __threadfence();
        named_bar(1, kEpiThreads);
        if (et == 0) {
          const uint32_t prev = atomicAdd(&a.counters[s.tile], 1u);
          *last_flag = (prev == (uint32_t)(s.nsegs - 1)) ? 1 : 0;
        }
        named_bar(1, kEpiThreads);
        if (*last_flag) {
          if (a.trace && et == 0) a.trace[c * 4 + 1] += 1ull << 32;
          __threadfence();
          const int c0 = c - s.seg;  // CTA of the tile's first segment
          const int tmax = min(TN, a.T - t0);
          for (int ch = 0; ch * kSlab < tmax; ++ch) {
            const int tl = ch * kSlab + tj;
            float acc[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] = 0.f;
            if (tl < tmax) {
              // fixed segment order (deterministic sums); the loads of four
              // segments are issued together so their latencies overlap
              for (int sg0 = 0; sg0 < s.nsegs; sg0 += 4) {
                float4 v[4][4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  const int sg = sg0 + u;
                  if (sg < s.nsegs) {
                    const float *slice = a.ws + ((size_t)(c0 + sg) * 2 + (sg == 0 ? 1 : 0)) * ((size_t)TN * BM);
                    const float4 *src = reinterpret_cast<const float4 *>(slice + (size_t)tl * BM + part * 16);
#pragma unroll
                    for (int j = 0; j < 4; ++j) v[u][j] = __ldcg(src + j);
                  }
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  if (sg0 + u < s.nsegs) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                      acc[4 * j] += v[u][j].x;
                      acc[4 * j + 1] += v[u][j].y;
                      acc[4 * j + 2] += v[u][j].z;
                      acc[4 * j + 3] += v[u][j].w;
                    }
                  }
                }
              }
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) slab[tj * kSlabPitch + part * 16 + j] = acc[j];
            named_bar(1, kEpiThreads);
            if (tl < tmax) write_row<EPI>(a, nt, t0 + tl, slab + tj * kSlabPitch, part, ll_e);
            named_bar(1, kEpiThreads);
          }
          if (et == 0) a.counters[s.tile] = 0u;
          if (EPI == kEpiAllReduce && !ll) publish_tile<TN>(p, s.tile, et);
          if (EPI == kEpiReduceScatter) publish_rows_rs<TN>(p, s.tile, 0, tmax, et);
          if (EPI == kEpiStore) finish_rows(p, t0, tmax, et, slab);
        }
        named_bar(1, kEpiThreads);  // last_flag is rewritten by the next segment
      }
    }
    if (a.trace && et == 0) {
      const unsigned long long te = ptx::globaltimer_ns();
      a.trace[c * 4 + 1] += te & 0xffffffffull;  // epilogue done (low 32 bits)
      *reinterpret_cast<volatile unsigned long long *>(slab) = te;
    }
    if (EPI == kEpiAllReduce) {
      if (ll)
        reduce_owned_chunks_ll<TN>(p, c, et, ll_e, slab);
      else
        reduce_owned_chunks<TN>(p, c, et, slab);
    }
  }

  // the producer and MMA warps ran their role on one elected lane: reconverge
  // each warp before the CTA-wide barrier (bar.sync is warp-aligned)
  __syncwarp();
  ptx::tc_fence_before();
  __syncthreads();
  if (a.trace && threadIdx.x == 0) {
    const unsigned long long te = *reinterpret_cast<volatile unsigned long long *>(slab);
    const unsigned long long tp = ptx::globaltimer_ns();
    a.trace[c * 4 + 2] = tp;
    if (te > tp) a.trace[c * 4 + 0] = 0;  // marks a barrier that did not order the epilogue
  }
  if (warp == 0) ptx::tmem_dealloc(tmem, C::TMEM_COLS);
  if (EPI == kEpiAllReduce && a.ll_state != nullptr && threadIdx.x == 0) ll_finish(a);
  if (a.trace && threadIdx.x == 0) a.trace[c * 4 + 3] = ptx::globaltimer_ns();
}

// ============================================================================
// Cluster split-K variant (decode shapes). The grid is G/CS clusters of CS
// CTAs; cluster k owns tiles k, k + G/CS, ... and its CTA r accumulates the
// K-blocks [r*kb/CS, (r+1)*kb/CS) of each in TMEM. The partial tiles are
// reduced through distributed shared memory inside the cluster: every CTA
// copies its accumulator to its own shared memory, signals its peers'
// mbarriers, and then sums one CS-th of the tile's tokens from all CS copies
// (in rank order: deterministic) and runs the epilogue on them. No partial
// ever leaves the GPC, so there is no global workspace, no counter and no
// serial fix-up at the end (which is what limits stream-K at these sizes).
template <int TN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_cluster_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                        const Params p) {
  using C = Cfg<TN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  uint8_t *stage_mem = base;
  float *slab = reinterpret_cast<float *>(base + S * C::STAGE_BYTES);
  float *red = reinterpret_cast<float *>(base + S * C::STAGE_BYTES + C::SLAB_BYTES);  // [TN][BM]
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + S * C::STAGE_BYTES + C::SLAB_BYTES + C::RED_BYTES);
  uint64_t *full = bars;
  uint64_t *empty = bars + S;
  uint64_t *acc_full = bars + 2 * S;       // [2]
  uint64_t *acc_empty = bars + 2 * S + 2;  // [2]
  uint64_t *red_ready = bars + 2 * S + 4;  // CS arrivals: every peer's partial is in place
  uint64_t *red_free = bars + 2 * S + 5;   // CS arrivals: every peer has read ours
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * S + 6);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const GemmArgs &a = p.a;
  const int CS = p.cs;
  const int rank = (int)ptx::cluster_ctarank();
  const int cid = blockIdx.x / CS;
  const int nclusters = gridDim.x / CS;
  const int kb0 = rank * p.kb / CS, kb1 = (rank + 1) * p.kb / CS;

  ptx::pdl_launch_dependents();
  if (a.trace && threadIdx.x == 0) a.trace[blockIdx.x * 4] = ptx::globaltimer_ns();
  if (warp == 0) {
    ptx::tmem_alloc(tmem_slot, C::TMEM_COLS);
    ptx::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&acc_full[i], 1);
      ptx::mbar_init(&acc_empty[i], kEpiThreads);
    }
    ptx::mbar_init(red_ready, CS);
    ptx::mbar_init(red_free, CS);
    ptx::fence_mbar_init();
  }
  if (threadIdx.x == 64) {
    ptx::prefetch_tmap(&tmW);
    ptx::prefetch_tmap(&tmX);
  }
  __syncwarp();
  ptx::tc_fence_before();
  ptx::cluster_sync_all();  // peers' barriers are initialised before any remote arrive
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ============================================================ producer
    if (ptx::elect_one()) {
      int pre = 0;  // weights of the first stages do not depend on the previous kernel
      for (int tile = cid; tile < p.tiles && pre < S; tile += nclusters) {
        const int nt = tile / p.t_tiles;
        for (int kb = kb0; kb < kb1 && pre < S; ++kb, ++pre) {
          ptx::mbar_arrive_expect_tx(&full[pre], C::STAGE_BYTES);
          ptx::tma_load_2d(stage_mem + pre * C::STAGE_BYTES, &tmW, &full[pre], kb * BK, nt * BM);
        }
      }
      ptx::pdl_wait();
      int i = 0;
      bool ok = true;
      for (int tile = cid; ok && tile < p.tiles; tile += nclusters) {
        const int nt = tile / p.t_tiles, tt = tile % p.t_tiles;
        if (a.x_ready) wait_rows_ready(a.x_ready, tt * TN, min(a.T, tt * TN + TN), a.status);
        for (int kb = kb0; kb < kb1; ++kb, ++i) {
          const int st = i % S;
          uint8_t *sm = stage_mem + st * C::STAGE_BYTES;
          if (i >= pre) {
            if (!ptx::mbar_wait(&empty[st], ((i / S) & 1) ^ 1, kWaitBudgetNs)) {
              report_status(a.status, kStatusMmaTimeout);
              ok = false;
              break;
            }
            ptx::mbar_arrive_expect_tx(&full[st], C::STAGE_BYTES);
            ptx::tma_load_2d(sm, &tmW, &full[st], kb * BK, nt * BM);
          }
          ptx::tma_load_2d(sm + C::W_BYTES, &tmX, &full[st], kb * BK, tt * TN);
        }
      }
    }
  } else if (warp == 1) {
    // ============================================================ MMA
    if (ptx::elect_one()) {
      constexpr uint32_t idesc = ptx::idesc_f16(BM, TN, /*bf16*/ 1, false, false);
      int i = 0, j = 0;
      bool ok = true;
      for (int tile = cid; ok && tile < p.tiles; tile += nclusters, ++j) {
        const int ab = j & 1;
        if (!ptx::mbar_wait(&acc_empty[ab], ((j >> 1) & 1) ^ 1, kWaitBudgetNs)) {
          report_status(a.status, kStatusEpilogueTimeout);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t acc = tmem + ab * C::ACC_COLS;
        for (int kb = kb0; kb < kb1; ++kb, ++i) {
          const int st = i % S;
          if (!ptx::mbar_wait(&full[st], (i / S) & 1, kWaitBudgetNs)) {
            report_status(a.status, kStatusTmaTimeout);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          uint8_t *sm = stage_mem + st * C::STAGE_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t da = ptx::smem_desc(sm + kk * 32, 16, 1024, ptx::kLayoutSW128);
            const uint64_t db = ptx::smem_desc(sm + C::W_BYTES + kk * 32, 16, 1024, ptx::kLayoutSW128);
            ptx::mma_f16_ss(acc, da, db, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          ptx::mma_commit(&empty[st]);
        }
        ptx::mma_commit(&acc_full[ab]);
      }
    }
  } else {
    // ============================================================ epilogue
    const int et = threadIdx.x - 64;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int tj = et / 8, part = et % 8;
    ptx::pdl_wait();
    const uint32_t ll_e = EPI == kEpiAllReduce ? ll_epoch(a) : 0u;
    const bool ll = EPI == kEpiAllReduce && a.ll_state != nullptr;
    const uint32_t red_addr = ptx::smem_u32(red);
    const uint32_t ready_addr = ptx::smem_u32(red_ready), free_addr = ptx::smem_u32(red_free);
    int j = 0;
    for (int tile = cid; tile < p.tiles; tile += nclusters, ++j) {
      const int ab = j & 1;
      const bool waited = ptx::mbar_wait(&acc_full[ab], (j >> 1) & 1, kWaitBudgetNs);
      if (!waited) report_status(a.status, kStatusEpilogueTimeout);
      ptx::tc_fence_after();
      const int nt = tile / p.t_tiles, tt = tile % p.t_tiles;
      const int t0 = tt * TN;
      const int tvalid = min(TN, a.T - t0);
      if (CS == 1) {
        // whole K in this CTA: straight to the epilogue
        for (int ch = 0; ch * kSlab < tvalid; ++ch) {
          uint32_t r[16];
          ptx::tmem_ld16(tmem + ab * C::ACC_COLS + ((uint32_t)(q * 32) << 16) + ch * kSlab, r);
          ptx::tmem_ld_wait();
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) slab[jj * kSlabPitch + row] = waited ? __uint_as_float(r[jj]) : 0.f;
          named_bar(1, kEpiThreads);
          const int t = t0 + ch * kSlab + tj;
          if (t < a.T) write_row<EPI>(a, nt, t, slab + tj * kSlabPitch, part, ll_e);
          named_bar(1, kEpiThreads);
        }
        ptx::tc_fence_before();
        ptx::mbar_arrive(&acc_empty[ab]);
        if (EPI == kEpiAllReduce && !ll) publish_rows<TN>(p, tile, 0, tvalid, et);
        if (EPI == kEpiReduceScatter) publish_rows_rs<TN>(p, tile, 0, tvalid, et);
        if (EPI == kEpiStore) finish_rows(p, t0, tvalid, et, slab);
        continue;
      }
      // our partial may overwrite `red` once every peer has read the previous one
      if (j > 0 && !ptx::mbar_wait_cluster(red_free, (j - 1) & 1, kWaitBudgetNs))
        report_status(a.status, kStatusPeerTimeout);
      for (int ch = 0; ch * kSlab < tvalid; ++ch) {
        uint32_t r[16];
        ptx::tmem_ld16(tmem + ab * C::ACC_COLS + ((uint32_t)(q * 32) << 16) + ch * kSlab, r);
        ptx::tmem_ld_wait();
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) red[(ch * kSlab + jj) * BM + row] = waited ? __uint_as_float(r[jj]) : 0.f;
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(&acc_empty[ab]);  // the MMA warp may start tile j + 2
      named_bar(1, kEpiThreads);
      if (et == 0)
        for (int s2 = 0; s2 < CS; ++s2) ptx::mbar_arrive_cluster(ptx::mapa_shared(ready_addr, s2));
      if (!ptx::mbar_wait_cluster(red_ready, j & 1, kWaitBudgetNs)) report_status(a.status, kStatusPeerTimeout);
      // sum our share of the tile's tokens over the CS partials, rank order
      const int lo = rank * tvalid / CS, hi = (rank + 1) * tvalid / CS;
      for (int b = lo; b < hi; b += kSlab) {
        const int tl = b + tj;
        float acc[16];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) acc[jj] = 0.f;
        if (tl < hi) {
          const uint32_t off = red_addr + (uint32_t)((tl * BM + part * 16) * 4);
          for (int s0 = 0; s0 < CS; s0 += 4) {
            float4 v[4][4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (s0 + u < CS) {
                const uint32_t src = ptx::mapa_shared(off, s0 + u);
#pragma unroll
                for (int x = 0; x < 4; ++x) v[u][x] = ptx::ld_dsmem_v4(src + 16 * x);
              }
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (s0 + u < CS) {
#pragma unroll
                for (int x = 0; x < 4; ++x) {
                  acc[4 * x] += v[u][x].x;
                  acc[4 * x + 1] += v[u][x].y;
                  acc[4 * x + 2] += v[u][x].z;
                  acc[4 * x + 3] += v[u][x].w;
                }
              }
          }
        }
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) slab[tj * kSlabPitch + part * 16 + jj] = acc[jj];
        named_bar(1, kEpiThreads);
        if (tl < hi) write_row<EPI>(a, nt, t0 + tl, slab + tj * kSlabPitch, part, ll_e);
        named_bar(1, kEpiThreads);
      }
      // every peer's partial has been read: release them
      named_bar(1, kEpiThreads);
      if (et == 0)
        for (int s2 = 0; s2 < CS; ++s2) ptx::mbar_arrive_cluster(ptx::mapa_shared(free_addr, s2));
      if (EPI == kEpiAllReduce && !ll) publish_rows<TN>(p, tile, lo, hi, et);
      if (EPI == kEpiReduceScatter) publish_rows_rs<TN>(p, tile, lo, hi, et);
      if (EPI == kEpiStore) finish_rows(p, t0 + lo, hi - lo, et, slab);
    }
    if (EPI == kEpiAllReduce) {
      if (ll)
        reduce_owned_chunks_ll<TN>(p, blockIdx.x, et, ll_e, slab);
      else
        reduce_owned_chunks<TN>(p, blockIdx.x, et, slab);
    }
  }

  __syncwarp();
  ptx::tc_fence_before();
  ptx::cluster_sync_all();  // no CTA leaves while a peer may still read its shared memory
  if (warp == 0) ptx::tmem_dealloc(tmem, C::TMEM_COLS);
  if (EPI == kEpiAllReduce && a.ll_state != nullptr && threadIdx.x == 0) ll_finish(a);
  if (a.trace && threadIdx.x == 0) a.trace[blockIdx.x * 4 + 3] = ptx::globaltimer_ns();
}

template <int TN, int EPI>
static void launch_tn(const CUtensorMap &tw, const CUtensorMap &tx, const Params &p,
                      cudaStream_t stream) {
  using C = Cfg<TN>;
  auto kern = gemm_kernel<TN, EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::smem(p.stages);
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kern, tw, tx, p);
}

// ---------------------------------------------------------------------------
// CTA-pair GEMM for prefill-sized calls (tcgen05.mma.cta_group::2, M = 256).
//
// A cluster of two CTAs owns one 256 x 256 output tile (256 weight rows x 256
// tokens): CTA r stages weight rows [128 r, 128 r + 128) and tokens
// [128 r, 128 r + 128) of the tile in its shared memory, the even CTA issues
// one M = 256, N = 256 MMA per 16-deep K step that reads both CTAs' stages,
// and each CTA's TMEM receives its 128 weight rows x all 256 tokens. Per SM
// that is 32 KB of operands per 2 x 128 x 256 x 64 multiply-adds, against
// 48 KB for the single-CTA 128 x 256 tile: a third less L2-to-SM traffic,
// which bounds the single-CTA kernel at prefill sizes. Two 256-column
// accumulators per CTA (all of TMEM) let each epilogue drain one tile while
// the MMA fills the next.
//
// Pipeline: both CTAs' producers load their halves with TMA (cta_group::2
// form: completion counted on the even CTA's stage barrier, no multicast);
// the even CTA's MMA thread releases each stage in both CTAs with one
// tcgen05.commit per CTA, and signals each CTA's accumulator likewise; both
// epilogues release an accumulator on the even CTA's barrier (256
// arrivals). Work units go to clusters round-robin: first the tiles of the
// full waves whole, then each tile of the last, partly filled wave as ps
// k-ranges, so that wave occupies ps times as many clusters. A k-range
// unit writes its fp32 partial to the workspace, counts itself on the
// tile's counter and waits (bounded) for the tile's other k-ranges: they
// are the first units of their clusters and the grid never exceeds the
// clusters that fit on the GPU, so all of them run at once. Each unit then
// sums 1/ps of the tile's token slabs over the ps partials, in split order
// (deterministic), and runs the epilogue on them: a CTA reads one tile's
// worth of partials whatever ps is.
constexpr int kPairTN = 256;
constexpr int kPairStages = 6;
constexpr int kPairHalf = BM * BK * 2;  // 128 rows x 64 bf16: one CTA's W or X half of a stage
constexpr int kPairStageBytes = 2 * kPairHalf;
constexpr int kPairAccCols = 256;
constexpr int kPairSmem = 1024 + kPairStages * kPairStageBytes + kSlab * kSlabPitch * 4 + 512;
static_assert(kPairSmem <= 232448, "pair GEMM shared memory");
constexpr int kPairMaxSplits = 8;    // k-ranges per tile of the last wave, at most
constexpr int kPairMinSplitKb = 8;   // k-blocks per k-range, at least
constexpr int kPairPartFloats = kPairTN * BM;  // one CTA's fp32 partial of a tile

// Unit u of a pair launch: tile, k-block range, and its index among the
// tile's k-ranges (-1: the whole tile). The k-range units come first (units
// [0, (tiles - pw) * ps) over the tiles [pw, tiles)): each is the first unit
// of its cluster, which makes the units of a tile co-resident, and their
// sums overlap the MMA of the cluster's next, whole tile (units from
// (tiles - pw) * ps on: tiles [0, pw)).
struct PairUnit {
  int tile, k0, k1, split;
};
__device__ __forceinline__ PairUnit pair_unit(const Params &p, int u, int kb, int tiles) {
  if (p.ps <= 1) return {u, 0, kb, -1};
  const int nsplit = (tiles - p.pw) * p.ps;
  if (u >= nsplit) return {u - nsplit, 0, kb, -1};
  const int s = u % p.ps;
  return {p.pw + u / p.ps, s * kb / p.ps, (s + 1) * kb / p.ps, s};
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                     const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *stage_mem = base;
  float *slab = reinterpret_cast<float *>(base + kPairStages * kPairStageBytes);
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + kPairStages * kPairStageBytes + kSlab * kSlabPitch * 4);
  uint64_t *full = bars;                              // [stages] (the even CTA's count both halves)
  uint64_t *empty = bars + kPairStages;               // [stages]
  uint64_t *acc_full = bars + 2 * kPairStages;        // [2]
  uint64_t *acc_empty = bars + 2 * kPairStages + 2;   // [2] (the even CTA's count both epilogues)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * kPairStages + 4);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = ptx::cluster_ctarank();
  const int pair = blockIdx.x / 2, npairs = gridDim.x / 2;
  const GemmArgs &a = p.a;
  const int t_tiles = (a.T + kPairTN - 1) / kPairTN;
  const int tiles = (a.N / (2 * BM)) * t_tiles;
  const int kb = a.K / BK;
  const int units = p.ps > 1 ? p.pw + (tiles - p.pw) * p.ps : tiles;
  // optional %globaltimer trace [grid][4]: entry, a k-range unit's tile
  // complete (all k-ranges arrived), its slice summed, exit
  if (a.trace && threadIdx.x == 0) a.trace[blockIdx.x * 4] = ptx::globaltimer_ns();
  auto on_even = [](uint64_t *b) { return ptx::mapa_shared(ptx::smem_u32(b), 0); };
  auto on_odd = [](uint64_t *b) { return ptx::mapa_shared(ptx::smem_u32(b), 1); };

  ptx::pdl_launch_dependents();
  if (warp == 0) {
    ptx::tmem_alloc_pair(tmem_slot, 2 * kPairAccCols);
    ptx::tmem_relinquish_pair();
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < kPairStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&acc_full[i], 1);
      ptx::mbar_init(&acc_empty[i], 2 * kEpiThreads);
    }
    ptx::fence_mbar_init();
  }
  if (threadIdx.x == 64) {
    ptx::prefetch_tmap(&tmW);
    ptx::prefetch_tmap(&tmX);
  }
  ptx::tc_fence_before();
  __syncwarp();
  __syncthreads();
  ptx::cluster_sync_all();  // both CTAs' barriers exist before any remote arrive or TMA completion
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ============================================================ producer (both CTAs)
    if (ptx::elect_one()) {
      ptx::pdl_wait();
      int i = 0;
      bool ok = true;
      for (int u = pair; ok && u < units; u += npairs) {
        const PairUnit pu = pair_unit(p, u, kb, tiles);
        const int mt = pu.tile / t_tiles, tt = pu.tile % t_tiles;
        for (int k = pu.k0; k < pu.k1; ++k, ++i) {
          const int s = i % kPairStages;
          if (!ptx::mbar_wait(&empty[s], ((i / kPairStages) & 1) ^ 1, kWaitBudgetNs)) {
            report_status(a.status, kStatusMmaTimeout);
            ok = false;
            break;
          }
          if (rank == 0) ptx::mbar_arrive_expect_tx(&full[s], 2 * kPairStageBytes);
          uint8_t *sm = stage_mem + s * kPairStageBytes;
          const uint32_t fb = on_even(&full[s]);
          ptx::tma_load_2d_pair(sm, &tmW, fb, k * BK, mt * 2 * BM + (int)rank * BM);
          ptx::tma_load_2d_pair(sm + kPairHalf, &tmX, fb, k * BK, tt * kPairTN + (int)rank * BM);
        }
      }
      // drain: every release the even CTA's MMA thread sends to this CTA's
      // stages has landed before the CTA may exit
      for (int j = i > kPairStages ? i - kPairStages : 0; ok && j < i; ++j)
        if (!ptx::mbar_wait(&empty[j % kPairStages], (j / kPairStages) & 1, kWaitBudgetNs)) {
          report_status(a.status, kStatusMmaTimeout);
          break;
        }
    }
  } else if (warp == 1) {
    // ============================================================ MMA (the even CTA)
    if (rank == 0 && ptx::elect_one()) {
      constexpr uint32_t idesc = ptx::idesc_f16(2 * BM, kPairTN, /*bf16*/ 1, false, false);
      int i = 0, n = 0;
      bool ok = true;
      for (int u = pair; ok && u < units; u += npairs, ++n) {
        const PairUnit pu = pair_unit(p, u, kb, tiles);
        const int ab = n & 1;
        if (!ptx::mbar_wait(&acc_empty[ab], ((n >> 1) & 1) ^ 1, kWaitBudgetNs)) {
          report_status(a.status, kStatusEpilogueTimeout);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t acc = tmem + ab * kPairAccCols;
        for (int k = pu.k0; k < pu.k1; ++k, ++i) {
          const int s = i % kPairStages;
          if (!ptx::mbar_wait(&full[s], (i / kPairStages) & 1, kWaitBudgetNs)) {
            report_status(a.status, kStatusTmaTimeout);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          uint8_t *sm = stage_mem + s * kPairStageBytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t da = ptx::smem_desc(sm + kk * 32, 16, 1024, ptx::kLayoutSW128);
            const uint64_t db = ptx::smem_desc(sm + kPairHalf + kk * 32, 16, 1024, ptx::kLayoutSW128);
            ptx::mma_f16_ss_pair(acc, da, db, idesc, (k > pu.k0 || kk > 0) ? 1u : 0u);
          }
          ptx::mma_commit_pair(on_even(&empty[s]));  // both CTAs' stage s may refill
          ptx::mma_commit_pair(on_odd(&empty[s]));
        }
        ptx::mma_commit_pair(on_even(&acc_full[ab]));  // both CTAs' accumulator ab is final
        ptx::mma_commit_pair(on_odd(&acc_full[ab]));
      }
    }
  } else {
    // ============================================================ epilogue (both CTAs)
    const int et = threadIdx.x - 64;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int tj = et / 8, part = et % 8;
    ptx::pdl_wait();
    int n = 0;
    for (int u = pair; u < units; u += npairs, ++n) {
      const PairUnit pu = pair_unit(p, u, kb, tiles);
      const int ab = n & 1;
      const bool waited = ptx::mbar_wait(&acc_full[ab], (n >> 1) & 1, kWaitBudgetNs);
      if (!waited) report_status(a.status, kStatusEpilogueTimeout);
      ptx::tc_fence_after();
      const int mt = pu.tile / t_tiles, tt = pu.tile % t_tiles;
      const int nt = mt * 2 + (int)rank;  // this CTA's 128-row weight tile
      const int t0 = tt * kPairTN;
      const int nch = min(kPairTN, a.T - t0 + kSlab - 1) / kSlab;  // slabs holding tokens
      const uint32_t acc_lane = tmem + ab * kPairAccCols + ((uint32_t)(q * 32) << 16);
      if (pu.split < 0) {
        for (int ch = 0; ch < nch; ++ch) {
          uint32_t r[16];
          ptx::tmem_ld16(acc_lane + ch * kSlab, r);
          ptx::tmem_ld_wait();
          if (!waited) {
#pragma unroll
            for (int j = 0; j < 16; ++j) r[j] = 0u;
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) slab[j * kSlabPitch + row] = __uint_as_float(r[j]);
          named_bar(1, kEpiThreads);
          const int t = t0 + ch * kSlab + tj;
          if (t < a.T) write_row<EPI>(a, nt, t, slab + tj * kSlabPitch, part);
          named_bar(1, kEpiThreads);
        }
        ptx::tc_fence_before();
        if (rank == 0)
          ptx::mbar_arrive(&acc_empty[ab]);
        else
          ptx::mbar_arrive_cluster(on_even(&acc_empty[ab]));
      } else {
        // k-range unit: this CTA's partial to its workspace slot as
        // [slab][4][row] float4 (4 tokens of a row per vector; a warp's
        // vectors are 512 contiguous bytes), then the accumulator is
        // released at once
        const int first = (pu.tile - p.pw) * p.ps;  // slot of the tile's k-range 0
        float4 *mine = reinterpret_cast<float4 *>(a.ws + ((size_t)(first + pu.split) * 2 + rank) * kPairPartFloats);
        for (int ch = 0; ch < nch; ++ch) {
          uint32_t r[16];
          ptx::tmem_ld16(acc_lane + ch * kSlab, r);
          ptx::tmem_ld_wait();
          if (!waited) {
#pragma unroll
            for (int j = 0; j < 16; ++j) r[j] = 0u;
          }
#pragma unroll
          for (int j4 = 0; j4 < 4; ++j4)
            __stcg(mine + (ch * 4 + j4) * BM + row,
                   make_float4(__uint_as_float(r[4 * j4]), __uint_as_float(r[4 * j4 + 1]),
                               __uint_as_float(r[4 * j4 + 2]), __uint_as_float(r[4 * j4 + 3])));
        }
        ptx::tc_fence_before();
        if (rank == 0)
          ptx::mbar_arrive(&acc_empty[ab]);
        else
          ptx::mbar_arrive_cluster(on_even(&acc_empty[ab]));
        __threadfence();  // the partial is visible before the arrival is counted
        named_bar(1, kEpiThreads);
        // [arrivals, departures] of this CTA's half of the tile
        uint32_t *cnt = a.counters + ((pu.tile - p.pw) * 2 + rank) * 2;
        if (et == 0) {
          // the tile's k-range units are the first units of their clusters
          // and the grid fits the GPU, so they all run at once: wait (bounded)
          // until every one has written its partial
          ptx::red_add_release_gpu(cnt, 1u);
          bool ok = ptx::ld_acquire_gpu(cnt) >= (uint32_t)p.ps;
          if (!ok) {
            const uint64_t start = ptx::globaltimer_ns();
            while (!ok) {
              for (int i = 0; i < 64 && !ok; ++i) ok = ptx::ld_acquire_gpu(cnt) >= (uint32_t)p.ps;
              if (!ok && ptx::globaltimer_ns() - start > kWaitBudgetNs) break;
            }
            if (!ok) report_status(a.status, kStatusEpilogueTimeout);
          }
          if (a.trace) a.trace[blockIdx.x * 4 + 1] = ptx::globaltimer_ns();
        }
        named_bar(1, kEpiThreads);
        __threadfence();
        // this unit sums slabs [c0, c1) of the tile over every k-range, in
        // split order (the same sum whichever unit does it), and runs the
        // epilogue on them
        const float4 *slot0 = reinterpret_cast<const float4 *>(a.ws + ((size_t)first * 2 + rank) * kPairPartFloats);
        constexpr size_t kSlotStride = 2 * (size_t)kPairPartFloats / 4;  // float4s from k-range s to s + 1
        const int c0 = pu.split * nch / p.ps, c1 = (pu.split + 1) * nch / p.ps;
        for (int ch = c0; ch < c1; ++ch) {
          // every k-range's four vectors in one round of independent loads
          float4 pv[kPairMaxSplits][4];
#pragma unroll
          for (int s2 = 0; s2 < kPairMaxSplits; ++s2)
#pragma unroll
            for (int j4 = 0; j4 < 4; ++j4)
              pv[s2][j4] = s2 < p.ps ? __ldcg(slot0 + s2 * kSlotStride + (ch * 4 + j4) * BM + row)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int j4 = 0; j4 < 4; ++j4) {
            float4 acc = pv[0][j4];
#pragma unroll
            for (int s2 = 1; s2 < kPairMaxSplits; ++s2) {
              if (s2 < p.ps) {
                acc.x += pv[s2][j4].x;
                acc.y += pv[s2][j4].y;
                acc.z += pv[s2][j4].z;
                acc.w += pv[s2][j4].w;
              }
            }
            slab[(4 * j4 + 0) * kSlabPitch + row] = acc.x;
            slab[(4 * j4 + 1) * kSlabPitch + row] = acc.y;
            slab[(4 * j4 + 2) * kSlabPitch + row] = acc.z;
            slab[(4 * j4 + 3) * kSlabPitch + row] = acc.w;
          }
          named_bar(1, kEpiThreads);
          const int t = t0 + ch * kSlab + tj;
          if (t < a.T) write_row<EPI>(a, nt, t, slab + tj * kSlabPitch, part);
          named_bar(1, kEpiThreads);
        }
        if (et == 0) {
          // the last unit to finish its sum zeroes both counters for the next call
          if (atomicAdd(cnt + 1, 1u) == (uint32_t)(p.ps - 1)) {
            cnt[0] = 0u;
            cnt[1] = 0u;
          }
          if (a.trace) a.trace[blockIdx.x * 4 + 2] = ptx::globaltimer_ns();
        }
      }
    }
  }

  __syncwarp();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync_all();  // the pair's MMAs, reads of TMEM and remote arrivals are done
  ptx::tc_fence_after();
  if (warp == 0) ptx::tmem_dealloc_pair(tmem, 2 * kPairAccCols);
  if (a.trace && threadIdx.x == 0) a.trace[blockIdx.x * 4 + 3] = ptx::globaltimer_ns();
}

// Clusters of two pair-GEMM CTAs that fit on the GPU at once.
template <int EPI>
static int pair_capacity() {
  static int cached = -1;
  if (cached >= 0) return cached;
  auto kern = gemm_pair_kernel<EPI>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 64);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kPairSmem;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cached = n;
  return n;
}

// The pair-GEMM launch of a call: clusters, whole tiles and k-ranges per
// tile of the last wave (np = 0: the single-CTA schedules). Taken for
// default-grid store / SwiGLU / RoPE+KV calls with N % 256 == 0 and
// T >= 256 whose 256 x 256 tiles keep at least 30 % of the resident clusters
// busy. The tiles of a last, partly filled wave are split into k-ranges
// (at most 8, each at least 8 k-blocks) so that the wave fills the
// clusters, when the workspace and counters hold their partials.
// Measured on B200 (us, L2 flushed; pair with k-ranges / pair with whole
// tiles / single-CTA stream-K / cuBLAS): T = 1536: o_proj 45 / 54 / 73 / 41,
// down_proj 121 / 151 / 205 / 117, gate_up 225 / 232 / 349 / 230;
// T = 512: down_proj 63 / 82 / 101; T = 256: o_proj 27 / 33 / 29,
// down_proj 47 / 80 / 62. SCHED_GEMM_PAIR=0 turns the kernel off, =1 takes
// it for every eligible shape; SCHED_GEMM_PAIR_SPLIT=0 keeps every tile
// whole.
struct PairPlan {
  int np = 0, whole = 0, splits = 1;
};

template <int EPI>
static PairPlan pair_plan_epi(const GemmArgs &a) {
  const char *v = std::getenv("SCHED_GEMM_PAIR");
  const int mode = v ? std::atoi(v) : -1;
  const char *vs = std::getenv("SCHED_GEMM_PAIR_SPLIT");
  const bool may_split = !(vs && std::atoi(vs) == 0);
  PairPlan none;
  if (mode == 0) return none;
  if (a.grid > 0 || a.norm_w != nullptr || a.x_ready != nullptr || a.N % (2 * BM) != 0 || a.K % BK != 0) return none;
  if (a.T < (mode == 1 ? 1 : 256)) return none;
  const long long tiles = (long long)(a.N / (2 * BM)) * ((a.T + kPairTN - 1) / kPairTN);
  const int cap = pair_capacity<EPI>();
  if (cap <= 0) return none;
  const long long full = tiles / cap, rem = tiles % cap;
  const int kb = a.K / BK;
  int S = 1;
  if (may_split && rem > 0) {
    S = (int)std::min<long long>(std::min<long long>(cap / rem, kb / kPairMinSplitKb), kPairMaxSplits);
    const long long need = rem * S * 2 * (long long)kPairPartFloats;
    if (S < 2 || a.ws == nullptr || a.counters == nullptr || need > a.ws_floats || 4 * rem > a.counter_count)
      S = 1;
  }
  PairPlan pl;
  double waves;  // in whole-tile times
  if (S > 1) {
    pl.whole = (int)(full * cap);
    pl.splits = S;
    pl.np = full > 0 ? cap : (int)(rem * S);
    waves = (double)full + 1.0 / S;
  } else {
    pl.whole = (int)tiles;
    pl.np = (int)std::min<long long>(cap, tiles);
    waves = (double)((tiles + cap - 1) / cap);
  }
  const double busy = (double)tiles / (waves * cap);  // resident clusters kept busy
  return (mode == 1 || busy >= 0.3) ? pl : none;
}

static PairPlan pair_plan(const GemmArgs &a) {
  switch (a.epi) {
    case kEpiStore: return pair_plan_epi<kEpiStore>(a);
    case kEpiSwiGLU: return pair_plan_epi<kEpiSwiGLU>(a);
    case kEpiRopeKV: return pair_plan_epi<kEpiRopeKV>(a);
    default: return PairPlan{};
  }
}

template <int EPI>
static void launch_pair(const CUtensorMap &tw, const CUtensorMap &tx, const Params &p, int npairs,
                        cudaStream_t stream) {
  auto kern = gemm_pair_kernel<EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmem);
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * npairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kPairSmem;
  cfg.stream = stream;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  cudaLaunchKernelEx(&cfg, kern, tw, tx, p);
}

template <int TN, int EPI>
static void launch_cluster_tn(const CUtensorMap &tw, const CUtensorMap &tx, const Params &p,
                              cudaStream_t stream) {
  using C = Cfg<TN>;
  auto kern = gemm_cluster_kernel<TN, EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::CSMEM);
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::CSMEM;
  cfg.stream = stream;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = p.cs;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  cudaLaunchKernelEx(&cfg, kern, tw, tx, p);
}

// Clusters of `cs` CTAs of this instantiation that fit on the GPU at once.
template <int TN, int EPI>
static int cluster_capacity(int cs) {
  using C = Cfg<TN>;
  static int cache[9] = {-1, -1, -1, -1, -1, -1, -1, -1, -1};
  if (cs < 1 || cs > 8) return 0;
  if (cache[cs] >= 0) return cache[cs];
  auto kern = gemm_cluster_kernel<TN, EPI>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::CSMEM);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cs * 64);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::CSMEM;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = cs;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache[cs] = n;
  return n;
}

// Cluster split-K plan of a call: cluster size and grid, or cs = 0 when the
// stream-K kernel is the better schedule. Cost model in K-blocks per CTA:
// cluster plan = rounds of tiles x K-blocks per rank (+2 for the DSMEM
// reduction), against the stream-K ideal units / SMs. Stream-K pays a serial
// global-memory fix-up per split tile on top of its ideal, which dominates
// when tiles are cut into two or more segments (tiles <= SMs / 2): there the
// cluster plan is taken within SCHED_GEMM_CLUSTER_SLACK (default 1.32) of
// the ideal; with more tiles only a near-perfect (<= 1.05) cluster plan is.
// (Measured on B200, Llama-3-8B decode shapes: o_proj and down_proj go to
// clusters, qkv and gate_up stay on stream-K.)
template <int TN, int EPI>
static void plan_cluster(Params &p, int num_sms) {
  p.cs = 0;
  static const double slack = [] {
    const char *v = std::getenv("SCHED_GEMM_CLUSTER_SLACK");
    return v ? std::atof(v) : 1.32;
  }();
  if (slack <= 0.0) return;
  const double ideal = (double)p.units / num_sms;
  double best = 1e30;
  int best_cs = 0, best_grid = 0;
  for (int cs = 1; cs <= 8; ++cs) {
    if (p.kb < cs) break;
    const int ncl = std::min(cluster_capacity<TN, EPI>(cs), num_sms / cs);
    if (ncl <= 0) continue;
    const int rounds = (p.tiles + ncl - 1) / ncl;
    const int used = std::min(ncl, p.tiles);
    const double cost = (double)rounds * ((p.kb + cs - 1) / cs) + (cs > 1 ? 2.0 : 0.0);
    if (cost < best - 1e-9) {
      best = cost;
      best_cs = cs;
      best_grid = used * cs;
    }
  }
  const double limit = (2 * p.tiles <= num_sms) ? slack : std::min(slack, 1.05);
  if (best_cs > 0 && best <= limit * ideal) {
    p.cs = best_cs;
    p.grid = best_grid;
  }
}

// Ring depth: the deepest that fits, unless SCHED_GEMM_SMEM_KB caps the
// shared memory of a CTA (a smaller CTA lets the next kernel's CTA become
// resident beside it and start its weight prefetch during this one's tail).
template <int TN>
// Without SCHED_GEMM_SMEM_KB, decode-width token tiles (TN <= 32) are capped
// at 128 KB: six or seven 18-20 KB stages still cover the weight stream, and
// the next kernel's CTA fits beside a finishing one (measured on B200: a
// batch-6 Llama-3-8B decode step 4.31 -> 4.23 ms and 4.38 -> 4.29 ms); wider
// tiles (prefill) keep the deepest ring, which their MMA rate needs.
static int stages_for() {
  using C = Cfg<TN>;
  static const int env_kb = [] {
    const char *v = std::getenv("SCHED_GEMM_SMEM_KB");
    return v ? std::atoi(v) : -1;
  }();
  const int cap_kb = env_kb >= 0 ? env_kb : (TN <= 32 ? 128 : 0);
  if (cap_kb <= 0) return C::STAGES;
  int s = C::STAGES;
  while (s > 2 && C::smem(s) > cap_kb * 1024) --s;
  return s;
}

template <int TN, int EPI>
static void launch_any(const CUtensorMap &tw, const CUtensorMap &tx, Params p, cudaStream_t stream) {
  if (p.cs > 0) {
    p.stages = Cfg<TN>::CSTAGES;
    launch_cluster_tn<TN, EPI>(tw, tx, p, stream);
  } else {
    p.stages = stages_for<TN>();
    launch_tn<TN, EPI>(tw, tx, p, stream);
  }
}

template <int EPI>
static void dispatch(int tn, const CUtensorMap &tw, const CUtensorMap &tx, Params p,
                     cudaStream_t stream) {
  switch (tn) {
    case 16: launch_any<16, EPI>(tw, tx, p, stream); break;
    case 32: launch_any<32, EPI>(tw, tx, p, stream); break;
    case 64: launch_any<64, EPI>(tw, tx, p, stream); break;
    case 128: launch_any<128, EPI>(tw, tx, p, stream); break;
    default: launch_any<256, EPI>(tw, tx, p, stream); break;
  }
}

// The cluster plan for the instantiation a call will use (TN <= 128; with
// the NVLink all-reduce epilogue each cluster rank pushes its share of the
// tile's tokens and releases the chunks it touched, see publish_rows).
template <int EPI>
static void plan_cluster_for(int tn, Params &p, int num_sms) {
  switch (tn) {
    case 16: plan_cluster<16, EPI>(p, num_sms); break;
    case 32: plan_cluster<32, EPI>(p, num_sms); break;
    case 64: plan_cluster<64, EPI>(p, num_sms); break;
    case 128: plan_cluster<128, EPI>(p, num_sms); break;
    default: p.cs = 0; break;
  }
}

// Token-tile width: the smallest of 16..256 that covers T; but when 256-wide
// tiles would leave SMs without a whole tile (N/128 x T/256 < SMs), 128-wide
// ones, which halve the stream-K splitting of every tile (measured on B200,
// T = 256: o_proj 62 -> 30 us, down_proj 85 -> 62 us; gate_up, with 224
// weight tiles, keeps 256). SCHED_GEMM_MAX_TN caps the width (default 256).
static int pick_tn(int T, int N, int num_sms) {
  static const int cap = [] {
    const char *v = std::getenv("SCHED_GEMM_MAX_TN");
    const int c = v ? std::atoi(v) : 256;
    return (c == 16 || c == 32 || c == 64 || c == 128) ? c : 256;
  }();
  int tn = 256;
  if (T <= 16) tn = 16;
  else if (T <= 32) tn = 32;
  else if (T <= 64) tn = 64;
  else if (T <= 128) tn = 128;
  const long long wide_tiles = (long long)(N / BM) * ((T + 255) / 256);
  if (tn == 256 && wide_tiles < (num_sms > 0 ? num_sms : 148)) tn = 128;
  return tn < cap ? tn : cap;
}

// Schedule of one call: grid, segments bound, whether tiles get split.
static void plan(const GemmArgs &a, Params &p, int &tn) {
  tn = pick_tn(a.T, a.N, a.num_sms);
  p.n_tiles = a.N / BM;
  p.t_tiles = (a.T + tn - 1) / tn;
  p.kb = a.K / BK;
  p.tiles = p.n_tiles * p.t_tiles;
  p.units = (long long)p.tiles * p.kb;
  int grid = a.grid > 0 ? a.grid : (a.num_sms > 0 ? a.num_sms : 148);
  // at least 4 k-blocks per CTA keeps the pipeline worth its set-up
  grid = (int)std::min<long long>(grid, std::max<long long>(1, p.units / 4));
  p.grid = std::max(1, grid);
}

static bool splits_tiles(const Params &p) {
  return p.units % p.grid != 0 || (p.units / p.grid) % p.kb != 0;
}

}  // namespace gemm

// Workspace floats a call of this shape needs (0 when no tile is split).
extern "C" long long sched_gemm_ws_floats(int T, int N, int K, int grid) {
  GemmArgs a{};
  a.T = T;
  a.N = N;
  a.K = K;
  a.grid = grid;
  gemm::Params p;
  int tn;
  gemm::plan(a, p, tn);
  if (!gemm::splits_tiles(p)) return 0;
  return (long long)p.grid * 2 * tn * gemm::BM;
}

namespace gemm {

// The schedule of a call: the stream-K plan for an explicit grid; for a
// default-grid call (grid <= 0), cluster split-K where it fits the shape and
// otherwise the stream-K plan. p.cs = 0 means stream-K.
static void final_plan(const GemmArgs &a, Params &p, int &tn) {
  plan(a, p, tn);
  p.cs = 0;
  if (a.grid > 0) return;
  const int sms = a.num_sms > 0 ? a.num_sms : 148;
  p.grid = std::max(1, sms);
  p.units = (long long)p.tiles * p.kb;
  if (a.epi == kEpiSwiGLU)
    plan_cluster_for<kEpiSwiGLU>(tn, p, sms);
  else if (a.epi == kEpiRopeKV)
    plan_cluster_for<kEpiRopeKV>(tn, p, sms);
  else if (a.epi == kEpiAllReduce)
    plan_cluster_for<kEpiAllReduce>(tn, p, sms);
  else if (a.epi == kEpiReduceScatter)
    plan_cluster_for<kEpiReduceScatter>(tn, p, sms);
  else
    plan_cluster_for<kEpiStore>(tn, p, sms);
  if (p.cs == 0) plan(a, p, tn);  // back to the stream-K grid
}

// Stream-K scratch a final plan needs: partial-slice floats and tile
// counters (both 0 when no tile is split, e.g. under cluster split-K).
static void scratch_need(const Params &p, int tn, long long &floats, int &counters) {
  floats = 0;
  counters = 0;
  if (p.cs == 0 && splits_tiles(p)) {
    floats = (long long)p.grid * 2 * tn * BM;
    counters = p.tiles;
  }
}

}  // namespace gemm

// The schedule sched_gemm_run would use for a default-grid call of this
// shape: writes the cluster size (0 = stream-K) and the grid.
extern "C" void sched_gemm_plan(int T, int N, int K, int epi, int num_sms, int *cs, int *grid) {
  GemmArgs a{};
  a.T = T;
  a.N = N;
  a.K = K;
  a.epi = epi;
  a.num_sms = num_sms;
  gemm::Params p;
  int tn;
  gemm::final_plan(a, p, tn);
  *cs = p.cs;
  *grid = p.grid;
}

// The CTA-pair launch sched_gemm_run would make for a default-grid call of
// this shape with a workspace of ws_floats floats and `counters` counters:
// clusters (0: a single-CTA schedule), whole tiles and k-ranges per tile of
// the last wave (1: none). Queries the device's cluster capacity.
extern "C" void sched_gemm_pair_plan(int T, int N, int K, int epi, long long ws_floats, int counters, int *np,
                                     int *whole, int *splits) {
  GemmArgs a{};
  a.T = T;
  a.N = N;
  a.K = K;
  a.epi = epi;
  static float dummy_ws;
  static uint32_t dummy_cnt;
  a.ws = ws_floats > 0 ? &dummy_ws : nullptr;
  a.ws_floats = ws_floats;
  a.counters = counters > 0 ? &dummy_cnt : nullptr;
  a.counter_count = counters;
  const gemm::PairPlan pl = gemm::pair_plan(a);
  *np = pl.np;
  *whole = pl.whole;
  *splits = pl.splits;
}

extern "C" int sched_gemm_run(const GemmArgs *args, cudaStream_t stream) {
  const GemmArgs &a = *args;
  if (a.T <= 0) return 0;
  if (a.N % gemm::BM != 0 || a.K % gemm::BK != 0) return -1;
  gemm::Params p;
  int tn;
  p.a = a;
  gemm::final_plan(a, p, tn);
  // the CTA-pair kernel sizes its k-ranges to the scratch it is given; the
  // stream-K scratch check applies to the single-CTA schedules only
  const gemm::PairPlan pl = gemm::pair_plan(a);
  long long need_floats;
  int need_counters;
  gemm::scratch_need(p, tn, need_floats, need_counters);
  if (pl.np == 0 && need_counters > 0) {
    if (a.ws == nullptr || a.counters == nullptr) return -2;
    if (need_floats > a.ws_floats || need_counters > a.counter_count) return -5;
  }
  if (a.epi == kEpiRopeKV && (a.N / gemm::BM != a.Hq + 2 * a.Hkv || a.cos_sin == nullptr ||
                              a.pos == nullptr || a.slot == nullptr))
    return -6;
  if (a.x_ready != nullptr && (reinterpret_cast<uintptr_t>(a.x_ready) & 15) != 0) return -7;
  if (a.norm_w != nullptr && (!(a.epi == kEpiStore || a.epi == kEpiAllReduce) || a.norm_res == nullptr ||
                              a.norm_out == nullptr || a.row_cnt == nullptr || a.y == nullptr || a.N % 8 != 0 ||
                              a.N > 16384 || a.ldy % 8 != 0))
    return -11;
  if (a.epi == kEpiAllReduce || a.epi == kEpiReduceScatter) {
    if (a.world < 1 || a.world > kMaxWorld || a.rank < 0 || a.rank >= a.world) return -7;
    const bool ll = a.epi == kEpiAllReduce && a.ll_state != nullptr;
    for (int j = 0; j < a.world; ++j) {
      if (a.recv[j] == nullptr || (a.flags[j] == nullptr && !ll)) return -7;
      if (ll && (reinterpret_cast<uintptr_t>(a.recv[j]) & 15) != 0) return -7;
    }
    // the low-latency line buffer holds [world][T][N / 4] lines per set
    if (ll && a.ll_set_lines < (long long)a.world * a.T * (a.N / 4)) return -7;
    if (a.ll_mc != nullptr && (!ll || (reinterpret_cast<uintptr_t>(a.ll_mc) & 15) != 0)) return -7;
  }
  try {
    CUtensorMap tw = tmap::make_2d(a.w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.N, a.K, a.K,
                                   gemm::BM, gemm::BK, CU_TENSOR_MAP_SWIZZLE_128B);
    if (pl.np > 0) {
      // CTA pairs: each CTA stages 128 of a tile's 256 tokens
      CUtensorMap tx2 = tmap::make_2d(a.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.T, a.K, a.ldx, gemm::BM,
                                      gemm::BK, CU_TENSOR_MAP_SWIZZLE_128B);
      p.pw = pl.whole;
      p.ps = pl.splits;
      const int np = pl.np;
      if (a.epi == kEpiSwiGLU)
        gemm::launch_pair<kEpiSwiGLU>(tw, tx2, p, np, stream);
      else if (a.epi == kEpiRopeKV)
        gemm::launch_pair<kEpiRopeKV>(tw, tx2, p, np, stream);
      else
        gemm::launch_pair<kEpiStore>(tw, tx2, p, np, stream);
      return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
    }
    CUtensorMap tx = tmap::make_2d(a.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.T, a.K, a.ldx, tn,
                                   gemm::BK, CU_TENSOR_MAP_SWIZZLE_128B);
    if (a.epi == kEpiSwiGLU)
      gemm::dispatch<kEpiSwiGLU>(tn, tw, tx, p, stream);
    else if (a.epi == kEpiAllReduce)
      gemm::dispatch<kEpiAllReduce>(tn, tw, tx, p, stream);
    else if (a.epi == kEpiReduceScatter)
      gemm::dispatch<kEpiReduceScatter>(tn, tw, tx, p, stream);
    else if (a.epi == kEpiRopeKV)
      gemm::dispatch<kEpiRopeKV>(tn, tw, tx, p, stream);
    else
      gemm::dispatch<kEpiStore>(tn, tw, tx, p, stream);
  } catch (const std::exception &) {
    return -3;
  }
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

// ---------------------------------------------------------------------------
// Fixed-scratch entry point (declared with its contract in gemm_api.h).
namespace gemm {

static __device__ __align__(256) float g_fixed_ws[kFixedScratchWsFloats];
static __device__ __align__(256) uint32_t g_fixed_counters[kFixedScratchCounters];

constexpr int kFixedMaxDevices = 64;
struct FixedScratch {
  float *ws = nullptr;
  uint32_t *counters = nullptr;
};
static std::mutex g_fixed_mu;
static FixedScratch g_fixed[kFixedMaxDevices];

// Device addresses of the arrays on the current device, looked up once.
static bool fixed_scratch(FixedScratch &out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kFixedMaxDevices) return false;
  std::lock_guard<std::mutex> lock(g_fixed_mu);
  FixedScratch &s = g_fixed[dev];
  if (s.ws == nullptr) {
    void *ws = nullptr, *cnt = nullptr;
    if (cudaGetSymbolAddress(&ws, g_fixed_ws) != cudaSuccess ||
        cudaGetSymbolAddress(&cnt, g_fixed_counters) != cudaSuccess) {
      cudaGetLastError();  // leave no sticky-looking error for the caller's next check
      return false;
    }
    s.ws = static_cast<float *>(ws);
    s.counters = static_cast<uint32_t *>(cnt);
  }
  out = s;
  return true;
}

}  // namespace gemm

extern "C" int sched_gemm_run_fixed_scratch(const GemmArgs *args, cudaStream_t stream) {
  if (args == nullptr || args->epi == kEpiAllReduce || args->epi == kEpiReduceScatter)
    return kFixedScratchBadEpilogue;
  GemmArgs a = *args;
  if (a.T <= 0) return 0;
  if (a.N % gemm::BM != 0 || a.K % gemm::BK != 0) return -1;
  gemm::FixedScratch s;
  if (!gemm::fixed_scratch(s)) return kFixedScratchLookupFailed;
  a.ws = s.ws;
  a.ws_floats = kFixedScratchWsFloats;
  a.counters = s.counters;
  a.counter_count = kFixedScratchCounters;
  // the capacity check runs on the schedule sched_gemm_run will launch: the
  // CTA-pair kernel sizes its k-ranges to this scratch, cluster split-K
  // needs none, stream-K needs its partial slices and tile counters
  if (gemm::pair_plan(a).np == 0) {
    gemm::Params p;
    int tn;
    gemm::final_plan(a, p, tn);
    long long need_floats;
    int need_counters;
    gemm::scratch_need(p, tn, need_floats, need_counters);
    if (need_floats > kFixedScratchWsFloats || need_counters > kFixedScratchCounters) return kFixedScratchTooLarge;
  }
  return sched_gemm_run(&a, stream);
}

extern "C" int sched_gemm_fixed_scratch_reset(cudaStream_t stream) {
  gemm::FixedScratch s;
  if (!gemm::fixed_scratch(s)) return kFixedScratchLookupFailed;
  // a memset node: no allocation, ordered on the caller's stream
  return cudaMemsetAsync(s.counters, 0, sizeof(uint32_t) * kFixedScratchCounters, stream) == cudaSuccess ? 0 : -4;
}
