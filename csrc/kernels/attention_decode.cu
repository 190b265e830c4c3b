// attention_decode.cu -- paged decode attention on the sm_100a tensor cores,
// with every scheduling lever of the manifest woven in at declared points.
//
// Problem: for each request b and KV head h, the G = Hq/Hkv query heads of h
// attend (one query token each) to the request's KV tokens, stored in
// 16-token pages addressed through a block table. The cache layout is
// [pages, Hkv, 16, 128] (one page of one head = 4 KB contiguous), so one 4-D
// TMA box (128-byte swizzle) fetches a whole page-head: TMA issue, not bytes,
// bounded the 2 KB half-page boxes used before (about 75 ns per box per SM).
//
// Tensor-core mapping ("transposed" decode): a decode query group is only G
// rows, far below the 128-row MMA, so the KV tokens take the M dimension:
//   S^T[128 tok x 16] = K_blk[128 tok x 128 d] . Q^T            (kind::f16)
//   O^T[128 d  x 16] = V_blk^T[128 d x 128 tok] . P^T[128 tok x 16]
// with the G heads padded to N = 16. S^T lands in TMEM with one token per
// lane, so each of the 128 softmax threads owns one token of the block; the
// PV result lands with one head-dimension row per lane, so the same thread
// owns one output row d and keeps its G running accumulators in registers.
//
// Warp roles (192 threads): warps 0-3 softmax + output (TMEM quarters 0-3),
// warp 4 TMA producer and task acquisition, warp 5 MMA issuer. KV blocks of
// 128 tokens flow through a STAGES-deep ring; S and O are double-buffered in
// TMEM and P in shared memory, so the S MMA of block i+1 and the PV MMA of
// block i run while the softmax of block i+1 is computed.
//
// Scheduling levers (sched/weave.cuh): tasks are (work item, KV head) with a
// work item = (request, KV range). A task is placed by pi (task =
// order[raw] with the order_size guard), observed by the timer (cycles added
// into timer[task]), truncated by shed (tokens at absolute position >= tau
// are dropped: exact truncated softmax, and the dropped KV is never read),
// and steered by the L2 policy (urgent tasks prefetch ahead and load with
// evict_last; polite tasks load with evict_first). Acquisition is static
// (grid = tasks), ticket (grid = workers, atomic counter that resets itself
// when the last worker exits), or cluster launch control (grid = tasks,
// idle CTAs steal unlaunched ones). The producer claims the next task right
// after it has issued the last load of the current one: late binding with
// a look-ahead of at most STAGES blocks.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>

#include "common.cuh"
#include "sched/ptx.cuh"
#include "sched/weave.cuh"
#include "tmap.h"

namespace attn {

constexpr int D = 128;
constexpr int PS = 16;                 // tokens per page
constexpr int BLK = 128;               // tokens per KV block (MMA M)
constexpr int PAGES_PER_BLK = BLK / PS;
constexpr int NPAD = 16;               // MMA N (query heads, padded)
constexpr int STAGES = 3;
// The MMA warp issues S = K.Q^T of block b+1 before O = V^T.P^T of block b,
// so two KV stages are in use at once: the ring needs at least two.
static_assert(STAGES >= 2, "the S/O issue order needs two KV stages in flight");
constexpr int kThreads = 192;
constexpr int kSoftmaxThreads = 128;
constexpr int HALF = BLK * 128;        // bytes of one 64-column half of a K or V block
constexpr int KV_BLOCK_BYTES = 2 * HALF;
// A K or V block in shared memory is 8 page-head boxes of 4 KB (one TMA box
// each, tmap::make_kv_pages): [row group][column half][8 rows][128 bytes], so
// an 8-row swizzle atom of one half is 1 KB, the other half's atom follows
// it, and consecutive 8-token atoms of one half are 2 KB apart.
constexpr int PAGE_BYTES = PS * 256;
constexpr int ATOM = 1024;
constexpr int ATOM_PAIR = 2048;
constexpr int STAGE_BYTES = 2 * KV_BLOCK_BYTES;  // K + V
constexpr int Q_BYTES = 2 * NPAD * 128;          // two 64-column halves of 16 rows
constexpr int P_BYTES = 2 * NPAD * 128;          // two 64-token halves of 16 rows
constexpr int TMEM_COLS = 64;  // S: cols [0,16) and [16,32) by block parity; O: [32,48) and [48,64) by task parity
constexpr float kRescaleLog2 = 8.f;  // a block moves a head's softmax reference only past 2^8
constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + Q_BYTES + 2 * P_BYTES + 1024;

struct Item {
  int32_t req;       // request (row of q/out and of the block table)
  int32_t kv_begin;  // first token of the range
  int32_t kv_end;    // one past the last token
  int32_t part;      // -1: write the final output; >= 0: partial slot for the merge
};

struct Params {
  const __nv_bfloat16 *q;  // [B, Hq, D]
  __nv_bfloat16 *out;      // [B, Hq, D]
  const int32_t *block_table;
  int bt_stride;
  const Item *items;
  int num_items;
  int num_tasks;  // num_items * Hkv
  int Hq, Hkv;
  float scale_log2;  // softmax scale * log2(e)
  float *part_o;     // [parts, Hq, D] (normalised partial outputs)
  float *part_lse;   // [parts, Hq] (log2-domain LSE)
  uint32_t *merge_cnt;  // [requests * Hkv] arrival counters (zero between calls), or null
  int splits;           // chunks per request when merging in-kernel (part = req * splits + s)
  int total_rows;       // rows of the cache tensor maps: pages * Hkv * 16 (an out-of-range row)
  int stage_split;      // block-table ids >= this name pages of the staging pool (tmK2/tmV2)
  int num_pages;        // pages of the device pool: ids in [num_pages, stage_split) are bad
  int stage_pages;      // pages of the staging pool: ids >= stage_split + stage_pages are bad
  SchedSlots slots;
  sched::PolicyConsts pc;
  int pf_blocks;  // urgent prefetch distance in KV blocks
  int *status;
  // L2 prefetch of the next kernel's operand (e.g. the output projection's
  // weights) while this kernel leaves DRAM mostly idle: each CTA issues bulk
  // prefetches for its 1/grid slice after its first task's loads (null: off)
  const uint8_t *l2_prefetch;
  long long l2_prefetch_bytes;
  // optional per-CTA %globaltimer trace [grid][8] (first task of a CTA):
  // entry, past set-up and the dependency wait, task published, its first
  // KV block's loads issued, first S tile seen by the softmax warps, last
  // block done, output / merge written, exit (nullptr: off)
  unsigned long long *trace;
};

struct TaskInfo {
  int32_t task;  // -1 = no more work
  int32_t req, kvh, kv_begin, kv_end, part, nblk, prio;  // prio: 0 none, 1 urgent, 2 polite
};

struct Shared {
  uint64_t k_full[STAGES], v_full[STAGES], kv_empty[STAGES];
  // pv_done[g & 1]: PV of global block g retired; o_free[task & 1]: the
  // softmax warps have read that task's O (its TMEM buffer may be reused)
  uint64_t s_ready[2], s_free[2], p_ready[2], pv_done[2], o_free[2];
  uint64_t q_ready, task_full[2], task_empty[2], clc_bar;
  alignas(16) uint4 clc_result;
  TaskInfo tasks[2];
  // per-warp partial max of a slow-path block and the flag that marks one
  // (grow_blk[g & 1] == g), double-buffered by block parity: block g+2
  // rewrites them only after every thread has passed block g+1's barrier,
  // i.e. finished reading block g's; per-warp partial l of a task, by task parity
  float red_max[2][4][NPAD];
  int grow_blk[2];
  float red_l[2][4][NPAD];
  uint32_t tmem_base;
  int merge_last;
};

// A block-table id names a device page [0, num_pages) or a staging page
// [stage_split, stage_split + stage_pages).
__device__ __forceinline__ bool page_ok(const Params &p, int page) {
  if (page < 0) return false;
  if (page >= p.stage_split) return page - p.stage_split < p.stage_pages;
  return page < p.num_pages;
}

__device__ __forceinline__ uint32_t swz(uint32_t row, uint32_t byte_in_row) {
  // 128-byte swizzle: the 16-byte chunk index is XORed with (row % 8).
  return row * 128u + ((((byte_in_row >> 4) ^ (row & 7u)) << 4) | (byte_in_row & 15u));
}

template <int G, bool WOVEN, int ACQ>
__global__ void __launch_bounds__(kThreads, 1)
    decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  const __grid_constant__ CUtensorMap tmK2, const __grid_constant__ CUtensorMap tmV2,
                  const Params p) {
  static_assert(G >= 1 && G <= NPAD, "group size");
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *stages = base;
  uint8_t *q_sm = base + STAGES * STAGE_BYTES;
  uint8_t *p_sm = q_sm + Q_BYTES;  // two buffers of P_BYTES
  Shared &sh = *reinterpret_cast<Shared *>(p_sm + 2 * P_BYTES);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const SchedSlots &sl = p.slots;

  // ------------------------------------------------------------------ setup
  unsigned long long *tr = p.trace != nullptr ? p.trace + (size_t)blockIdx.x * 8 : nullptr;
  if (tr != nullptr && threadIdx.x == 0) tr[0] = ptx::globaltimer_ns();
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
      sh.grow_blk[i] = -1;
      ptx::mbar_init(&sh.o_free[i], kSoftmaxThreads);
      ptx::mbar_init(&sh.task_full[i], 1);
      ptx::mbar_init(&sh.task_empty[i], 1 + kSoftmaxThreads);
    }
    ptx::mbar_init(&sh.q_ready, kSoftmaxThreads);
    ptx::mbar_init(&sh.clc_bar, 1);
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tmK);
    ptx::prefetch_tmap(&tmV);
  }
  // Q and P rows >= G are MMA padding and must be zero; they are never
  // written afterwards. (KV rows past a request's last page come from
  // out-of-range TMA boxes, which the hardware fills with zeros.)
  if (WOVEN) sched::pdl_launch_dependents();
  {
    uint4 z = make_uint4(0, 0, 0, 0);
    uint4 *b4 = reinterpret_cast<uint4 *>(q_sm);
    const int n16 = (Q_BYTES + 2 * P_BYTES) / 16;
    for (int i = threadIdx.x; i < n16; i += kThreads) b4[i] = z;
  }
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_before();
  __syncwarp();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = sh.tmem_base;

  // Launch-wide acquisition decision (uniform across the grid).
  uint32_t wq_tasks = (WOVEN && ACQ != (int)sched::Acquire::Static) ? sched::wq_num_tasks(sl) : 0u;
  const bool dynamic = wq_tasks != 0u;
  const uint32_t ntasks = dynamic ? min(wq_tasks, (uint32_t)p.num_tasks) : (uint32_t)p.num_tasks;

  // A task's table reads (order, item, budget, policy) and its page ids
  // touch only tables the host wrote before the step, never the previous
  // kernel's output (q and the newest KV rows), so the producer resolves its
  // first task and that task's first page ids before waiting for the
  // previous kernel: three dependent loads leave the critical path.
  auto build_task = [&](uint32_t raw) -> TaskInfo {
    TaskInfo ti;
    ti.task = -1;
    if (raw < ntasks) {
      uint32_t task = WOVEN ? sched::remap(sl, raw, ntasks) : raw;
      const int item = task / p.Hkv;
      const Item it = p.items[item];
      ti.task = (int32_t)task;
      ti.req = it.req;
      ti.kvh = task % p.Hkv;
      ti.kv_begin = it.kv_begin;
      int kv_end = it.kv_end;
      ti.prio = 0;
      if (WOVEN) {
        const uint32_t tau = sched::budget(sl, task);
        if (tau != 0xFFFFFFFFu) kv_end = min(kv_end, (int)tau);
        const sched::PolicyFlags pf = sched::policy(sl, task, p.pc);
        ti.prio = pf.urgent ? 1 : (pf.polite ? 2 : 0);
      }
      ti.kv_end = max(kv_end, it.kv_begin);
      ti.part = it.part;
      ti.nblk = (ti.kv_end - ti.kv_begin + BLK - 1) / BLK;
    }
    return ti;
  };
  TaskInfo first_ti;
  first_ti.task = -1;
  int first_ids[PAGES_PER_BLK];
  if (warp == 4 && lane == 0) {
    first_ti = build_task(blockIdx.x);
    if (first_ti.task >= 0 && first_ti.nblk > 0) {
      const int32_t *bt = p.block_table + (size_t)first_ti.req * p.bt_stride;
      const int pg0 = first_ti.kv_begin / PS;
      const int npg = min(PAGES_PER_BLK, (first_ti.kv_end + PS - 1) / PS - pg0);
#pragma unroll
      for (int pi = 0; pi < PAGES_PER_BLK; ++pi) first_ids[pi] = pi < npg ? __ldg(bt + pg0 + pi) : -1;
    }
  }

  if (WOVEN) sched::pdl_wait();
  if (tr != nullptr && threadIdx.x == 0) tr[1] = ptx::globaltimer_ns();

  if (warp == 4) {
    // ============================================================ producer
    if (lane == 0) {
      uint32_t raw = blockIdx.x;
      uint32_t clc_phase = 0;
      int blk_counter = 0;  // global KV block counter of this CTA (ring position)
      int j = 0;            // task counter of this CTA
      const uint64_t pol_last = ptx::policy_evict_last();
      const uint64_t pol_first = ptx::policy_evict_first();
      bool stop = false;
      while (!stop) {
        TaskInfo ti = j == 0 ? first_ti : build_task(raw);
        // publish the task to the MMA and softmax warps
        const int slot = j & 1;
        if (!ptx::mbar_wait(&sh.task_empty[slot], ((j >> 1) & 1) ^ 1, kWaitBudgetNs)) {
          report_timeout(p.status, kStatusEpilogueTimeout, kWaitProducerTaskEmpty);
          ti.task = -1;
        }
        sh.tasks[slot] = ti;
        ptx::mbar_arrive(&sh.task_full[slot]);
        ++j;
        if (tr != nullptr && j == 1) tr[2] = ptx::globaltimer_ns();
        if (ti.task < 0) break;

        // stream the task's KV blocks
        const int32_t *bt = p.block_table + (size_t)ti.req * p.bt_stride;
        const int first_page = ti.kv_begin / PS;  // kv_begin is block-aligned
        const int last_page = (ti.kv_end + PS - 1) / PS;
        // The page ids of a block are loaded together (independent loads, so
        // their latencies overlap) and one block ahead of its TMA issue, so
        // the block-table reads hide behind the wait for a free stage
        // instead of adding eight load latencies to every block.
        int ids_next[PAGES_PER_BLK];
        auto load_ids = [&](int b, int *ids) {
          const int pg0 = first_page + b * PAGES_PER_BLK;
          const int npg = min(PAGES_PER_BLK, last_page - pg0);
#pragma unroll
          for (int pi = 0; pi < PAGES_PER_BLK; ++pi) ids[pi] = pi < npg ? __ldg(bt + pg0 + pi) : -1;
        };
        if (ti.nblk > 0) {
          if (j == 1) {  // the first task's ids were loaded before the dependency wait
#pragma unroll
            for (int pi = 0; pi < PAGES_PER_BLK; ++pi) ids_next[pi] = first_ids[pi];
          } else {
            load_ids(0, ids_next);
          }
        }
        for (int b = 0; b < ti.nblk; ++b, ++blk_counter) {
          int ids[PAGES_PER_BLK];
#pragma unroll
          for (int pi = 0; pi < PAGES_PER_BLK; ++pi) ids[pi] = ids_next[pi];
          if (b + 1 < ti.nblk) load_ids(b + 1, ids_next);
          const int s = blk_counter % STAGES;
          const uint32_t ph = (blk_counter / STAGES) & 1;
          if (!ptx::mbar_wait(&sh.kv_empty[s], ph ^ 1, kWaitBudgetNs)) {
            report_status(p.status, kStatusMmaTimeout);
            stop = true;
            break;
          }
          uint8_t *kst = stages + s * STAGE_BYTES;
          uint8_t *vst = kst + KV_BLOCK_BYTES;
          const int pg0 = first_page + b * PAGES_PER_BLK;
          const int npg = min(PAGES_PER_BLK, last_page - pg0);
          ptx::mbar_arrive_expect_tx(&sh.k_full[s], KV_BLOCK_BYTES);
          ptx::mbar_arrive_expect_tx(&sh.v_full[s], KV_BLOCK_BYTES);
          // one 4 KB box per page-head (row group = row / 8, two per page);
          // pages past the request's end: an out-of-range box reads zeros;
          // ids from stage_split on live in the staging pool (tiered KV)
          auto page_box = [&](int pi, int &rg, bool &staged) {
            int page = ids[pi];
            if (pi < npg && !page_ok(p, page)) {  // reported; read as an out-of-range (zero) box
              report_bad_index(p.status, kSiteDecodePage, page);
              page = -1;
            }
            staged = page >= p.stage_split;
            rg = page < 0 ? p.total_rows / 8
                          : ((staged ? page - p.stage_split : page) * p.Hkv + ti.kvh) * (PS / 8);
          };
          // The hint decision is taken once per block, outside the page loop:
          // a per-page branch inside the unrolled loop made the woven kernel
          // stream KV 24 % slower than the stock one (measured on B200) even
          // for tasks without a hint.
          if (!(WOVEN && ti.prio != 0)) {
#pragma unroll
            for (int pi = 0; pi < PAGES_PER_BLK; ++pi) {
              int rg;
              bool staged;
              page_box(pi, rg, staged);
              ptx::tma_load_4d(kst + pi * PAGE_BYTES, staged ? &tmK2 : &tmK, &sh.k_full[s], 0, 0, 0, rg);
              ptx::tma_load_4d(vst + pi * PAGE_BYTES, staged ? &tmV2 : &tmV, &sh.v_full[s], 0, 0, 0, rg);
            }
          } else {
            const uint64_t pol = ti.prio == 1 ? pol_last : pol_first;
#pragma unroll
            for (int pi = 0; pi < PAGES_PER_BLK; ++pi) {
              int rg;
              bool staged;
              page_box(pi, rg, staged);
              ptx::tma_load_4d_hint(kst + pi * PAGE_BYTES, staged ? &tmK2 : &tmK, &sh.k_full[s], 0, 0, 0, rg, pol);
              ptx::tma_load_4d_hint(vst + pi * PAGE_BYTES, staged ? &tmV2 : &tmV, &sh.v_full[s], 0, 0, 0, rg, pol);
            }
            // urgent: warm L2 with the pages pf_blocks ahead (pure hint)
            if (ti.prio == 1 && p.pf_blocks > 0) {
              const int pf0 = pg0 + p.pf_blocks * PAGES_PER_BLK;
              const int pfn = min(PAGES_PER_BLK, last_page - pf0);
              for (int pi = 0; pi < pfn; ++pi) {
                const int page = __ldg(bt + pf0 + pi);
                if (!page_ok(p, page)) continue;
                const bool staged = page >= p.stage_split;
                const int rg = ((staged ? page - p.stage_split : page) * p.Hkv + ti.kvh) * (PS / 8);
                const CUtensorMap *mk = staged ? &tmK2 : &tmK;
                const CUtensorMap *mv = staged ? &tmV2 : &tmV;
                ptx::tma_prefetch_4d(mk, 0, 0, 0, rg);
                ptx::tma_prefetch_4d(mv, 0, 0, 0, rg);
              }
            }
          }
          if (tr != nullptr && j == 1 && b == 0) tr[3] = ptx::globaltimer_ns();
          if (j == 1 && b == 0 && p.l2_prefetch != nullptr) {
            // this CTA's 16-byte-aligned slice of the next operand, in chunks
            const long long per = ((p.l2_prefetch_bytes / gridDim.x) + 15) & ~15ll;
            const long long lo = per * blockIdx.x;
            const long long hi = min(p.l2_prefetch_bytes & ~15ll, lo + per);
            for (long long o = lo; o < hi; o += 65536) {
              const uint32_t n = (uint32_t)min(65536ll, hi - o);
              asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p.l2_prefetch + o), "r"(n)
                           : "memory");
            }
          }
        }
        if (stop) {
          // tell the consumers there is nothing more
          const int s2 = j & 1;
          if (ptx::mbar_wait(&sh.task_empty[s2], ((j >> 1) & 1) ^ 1, kWaitBudgetNs)) {
            TaskInfo none;
            none.task = -1;
            sh.tasks[s2] = none;
            ptx::mbar_arrive(&sh.task_full[s2]);
          }
          break;
        }
        // acquire the next task (late binding: after this task's last load)
        if (!dynamic) {
          raw += gridDim.x;  // static: grid-stride (one task per CTA when grid == tasks)
        } else if (ACQ == (int)sched::Acquire::Ticket) {
          raw = sl.queue != nullptr ? gridDim.x + sched::claim_ticket(sl) : ntasks;
        } else if (ACQ == (int)sched::Acquire::Clc) {
          bool to = false;
          raw = sched::claim_clc(&sh.clc_result, &sh.clc_bar, clc_phase, ntasks,
                                 kWaitBudgetNs, &to);
          if (to) report_status(p.status, kStatusClcTimeout);
        }
      }
    }
  } else if (warp == 5) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = ptx::idesc_f16(BLK, NPAD, 1, false, false);  // K-major A, K-major B
      constexpr uint32_t idO = ptx::idesc_f16(D, NPAD, 1, true, false);     // MN-major A (V^T)
      int blk = 0;  // global block counter
      int j = 0;
      int o_use[2] = {0, 0};  // tasks with KV blocks that used each O buffer
      int q_use = 0;          // tasks with KV blocks (q_ready phases)
      bool ok = true;
      while (ok) {
        const int slot = j & 1;
        if (!ptx::mbar_wait(&sh.task_full[slot], (j >> 1) & 1, kWaitBudgetNs)) {
          report_timeout(p.status, kStatusEpilogueTimeout, kWaitMmaTaskFull);
          break;
        }
        const TaskInfo ti = sh.tasks[slot];
        ++j;
        if (ti.task < 0) break;
        // Q of this task is written by the softmax warps (only for tasks with
        // KV blocks, counted here the same way, so the barrier cannot run a
        // phase ahead of this wait)
        if (ti.nblk > 0) {
          if (!ptx::mbar_wait(&sh.q_ready, q_use & 1, kWaitBudgetNs)) {
            report_timeout(p.status, kStatusEpilogueTimeout, kWaitMmaQReady);
            break;
          }
          ++q_use;
        }
        auto issue_s = [&](int g) -> bool {  // g: global block index
          const int s = g % STAGES;
          const int sb = g & 1;
          if (!ptx::mbar_wait(&sh.k_full[s], (g / STAGES) & 1, kWaitBudgetNs)) return false;
          if (!ptx::mbar_wait(&sh.s_free[sb], ((g >> 1) & 1) ^ 1, kWaitBudgetNs)) return false;
          ptx::tc_fence_after();
          const uint8_t *kst = stages + s * STAGE_BYTES;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            // K block: 8-token atoms of one column half 2048 bytes apart (SBO), the
            // other half at +1024
            const uint8_t *a = kst + (kk / 4) * ATOM + (kk % 4) * 32;
            const uint8_t *b = q_sm + (kk / 4) * (NPAD * 128) + (kk % 4) * 32;
            ptx::mma_f16_ss(tmem + sb * 16, ptx::smem_desc(a, 16, ATOM_PAIR, ptx::kLayoutSW128),
                            ptx::smem_desc(b, 16, 1024, ptx::kLayoutSW128), idS, kk > 0);
          }
          ptx::mma_commit(&sh.s_ready[sb]);
          return true;
        };
        // this task's O buffer (by task parity). Only tasks with KV blocks
        // use it: the softmax warps release it after reading O, which they
        // cannot do before this wait since they need this task's PV products.
        // (A task without blocks is finished by the softmax warps without
        // the MMA warp, so counting it would let the barrier run a phase ahead.)
        const int ot = (j - 1) & 1;
        if (ti.nblk > 0) {
          if (!ptx::mbar_wait(&sh.o_free[ot], (o_use[ot] & 1) ^ 1, kWaitBudgetNs)) {
            report_timeout(p.status, kStatusEpilogueTimeout, kWaitMmaOFree);
            break;
          }
          ++o_use[ot];
        }
        auto issue_o = [&](int g, bool first) -> bool {
          const int s = g % STAGES;
          const int ob = g & 1;
          if (!ptx::mbar_wait(&sh.v_full[s], (g / STAGES) & 1, kWaitBudgetNs)) return false;
          if (!ptx::mbar_wait(&sh.p_ready[ob], (g >> 1) & 1, kWaitBudgetNs)) return false;
          ptx::tc_fence_after();
          const uint8_t *vst = stages + s * STAGE_BYTES + KV_BLOCK_BYTES;
          const uint8_t *pb = p_sm + ob * P_BYTES;
#pragma unroll
          for (int kk = 0; kk < BLK / 16; ++kk) {
            // A = V^T, MN-major: 64 d per 128-byte row, other d-half at +1024 (LBO),
            // 8-token groups at +2048 (SBO); 16 tokens per MMA = +4096 bytes.
            const uint8_t *a = vst + kk * 2 * ATOM_PAIR;
            const uint8_t *b = pb + (kk / 4) * (NPAD * 128) + (kk % 4) * 32;
            ptx::mma_f16_ss(tmem + 32 + ot * 16, ptx::smem_desc(a, ATOM, ATOM_PAIR, ptx::kLayoutSW128),
                            ptx::smem_desc(b, 16, 1024, ptx::kLayoutSW128), idO, (!first || kk > 0) ? 1u : 0u);
          }
          ptx::mma_commit(&sh.pv_done[ob]);
          ptx::mma_commit(&sh.kv_empty[s]);
          return true;
        };
        const int g0 = blk;
        if (ti.nblk > 0 && !issue_s(g0)) ok = false;
        for (int b = 0; ok && b < ti.nblk; ++b) {
          if (b + 1 < ti.nblk && !issue_s(g0 + b + 1)) { ok = false; break; }
          if (!issue_o(g0 + b, b == 0)) { ok = false; break; }
        }
        if (!ok) report_status(p.status, kStatusTmaTimeout);
        blk += ti.nblk;
        ptx::mbar_arrive(&sh.task_empty[slot]);
      }
    }
  } else {
    // ============================================================ softmax + output
    const int t = threadIdx.x;  // 0..127: token row of S^T, d row of O^T
    const int q4 = warp;        // TMEM lane quarter
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    int blk = 0;
    int j = 0;
    // the timer's off-flag is read once per CTA, at entry (it decides this
    // launch's writes)
    const bool timer_off = WOVEN ? sched::timer_off_at_entry(sl) : true;
    while (true) {
      const int slot = j & 1;
      if (!ptx::mbar_wait(&sh.task_full[slot], (j >> 1) & 1, kWaitBudgetNs)) {
        report_timeout(p.status, kStatusEpilogueTimeout, kWaitSoftmaxTaskFull);
        break;
      }
      const TaskInfo ti = sh.tasks[slot];
      ++j;
      if (ti.task < 0) break;
      const unsigned long long t0 = sched::clock_now();

      // Q rows of this task -> swizzled K-major tile (rows >= G stay zero);
      // a task without KV blocks issues no MMA and needs none
      if (ti.nblk > 0) {
        if (t < G * 16) {
          const int h = t / 16, c = t % 16;
          const uint4 v = __ldg(reinterpret_cast<const uint4 *>(
              p.q + ((size_t)ti.req * p.Hq + ti.kvh * G + h) * D) + c);
          *reinterpret_cast<uint4 *>(q_sm + (c / 8) * (NPAD * 128) + swz(h, (c % 8) * 16)) = v;
        }
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(&sh.q_ready);
      }

      // Online softmax with a fixed reference per head: every block whose
      // scores stay within 2^8 of the reference m uses P = 2^(s - m), so the
      // P of all blocks of a task share one m, O accumulates in TMEM across
      // the task's blocks (no per-block fold), and each thread keeps the sum
      // of its own token's P (one reduction per task). A block that raises a
      // head's max by more than 2^8 (the first block always does) takes the
      // CTA-uniform slow path: exact block max, new reference, O and the
      // partial sums scaled. Normal blocks cost one barrier and no shuffles.
      const int ot = (j - 1) & 1;  // this task's O buffer: TMEM columns 32 + 16 ot
      const uint32_t o_col = 32 + ot * 16;
      float m_ref[G], l_t[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        m_ref[h] = -INFINITY;
        l_t[h] = 0.f;
      }
      bool ok = true;
      for (int b = 0; b < ti.nblk; ++b) {
        const int g = blk + b;
        const int sb = g & 1;
        if (!ptx::mbar_wait(&sh.s_ready[sb], (g >> 1) & 1, kWaitBudgetNs)) {
          report_status(p.status, kStatusMmaTimeout);
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        if (tr != nullptr && j == 1 && b == 0 && t == 0) tr[4] = ptx::globaltimer_ns();
        uint32_t sr[16];
        ptx::tmem_ld16(tmem + lane_off + sb * 16, sr);
        ptx::tmem_ld_wait();
        ptx::tc_fence_before();
        ptx::mbar_arrive(&sh.s_free[sb]);
        const int tok = ti.kv_begin + b * BLK + t;
        const bool valid = tok < ti.kv_end;
        float s[G];
        bool grow = false;
#pragma unroll
        for (int h = 0; h < G; ++h) {
          s[h] = valid ? __uint_as_float(sr[h]) * p.scale_log2 : -INFINITY;
          grow |= s[h] > m_ref[h] + kRescaleLog2;
        }
        if (__any_sync(0xffffffffu, grow) && lane == 0) sh.grow_blk[sb] = g;
        named_bar(1, kSoftmaxThreads);
        if (sh.grow_blk[sb] == g) {  // CTA-uniform slow path
#pragma unroll
          for (int h = 0; h < G; ++h) {
            float v = s[h];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
            if (lane == 0) sh.red_max[sb][q4][h] = v;
          }
          named_bar(1, kSoftmaxThreads);
          float alpha[G];
          bool scaled = false;  // the same in every thread: computed from shared values
#pragma unroll
          for (int h = 0; h < G; ++h) {
            const float(&rm)[4][NPAD] = sh.red_max[sb];
            const float bm = fmaxf(fmaxf(rm[0][h], rm[1][h]), fmaxf(rm[2][h], rm[3][h]));
            alpha[h] = 1.f;
            if (bm > m_ref[h] + kRescaleLog2) {
              alpha[h] = m_ref[h] == -INFINITY ? 0.f : ex2_approx(m_ref[h] - bm);
              m_ref[h] = bm;
              scaled = true;
            }
            l_t[h] *= alpha[h];
          }
          if (scaled && b > 0) {
            // O holds blocks [0, b) of this task: scale each head's column
            // once PV(g-1) has completed
            const int gp = g - 1;
            if (!ptx::mbar_wait(&sh.pv_done[gp & 1], (gp >> 1) & 1, kWaitBudgetNs)) {
              report_status(p.status, kStatusMmaTimeout);
              ok = false;
              break;
            }
            ptx::tc_fence_after();
            uint32_t o[16];
            ptx::tmem_ld16(tmem + lane_off + o_col, o);
            ptx::tmem_ld_wait();
#pragma unroll
            for (int h = 0; h < G; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * alpha[h]);
            ptx::tmem_st16(tmem + lane_off + o_col, o);
            ptx::tmem_st_wait();
          }
        }
        // P^T -> shared (bf16, swizzled K-major, row = head, column = token)
        uint8_t *pb = p_sm + sb * P_BYTES + (t / 64) * (NPAD * 128);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float pr = s[h] == -INFINITY ? 0.f : ex2_approx(s[h] - m_ref[h]);
          l_t[h] += pr;
          *reinterpret_cast<__nv_bfloat16 *>(pb + swz(h, (t % 64) * 2)) = __float2bfloat16(pr);
        }
        ptx::fence_proxy_async_smem();
        ptx::tc_fence_before();
        ptx::mbar_arrive(&sh.p_ready[sb]);
      }
      // l per head: the 128 threads' partial sums (warp, then the 4 warps)
      float m_run[G], l_run[G], o_acc[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float v = l_t[h];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) sh.red_l[ot][q4][h] = v;
        m_run[h] = m_ref[h];
        o_acc[h] = 0.f;
      }
      named_bar(1, kSoftmaxThreads);
#pragma unroll
      for (int h = 0; h < G; ++h)
        l_run[h] = (sh.red_l[ot][0][h] + sh.red_l[ot][1][h]) + (sh.red_l[ot][2][h] + sh.red_l[ot][3][h]);
      if (ok && ti.nblk > 0) {
        const int gl = blk + ti.nblk - 1;
        if (ptx::mbar_wait(&sh.pv_done[gl & 1], (gl >> 1) & 1, kWaitBudgetNs)) {
          ptx::tc_fence_after();
          uint32_t orr[16];
          ptx::tmem_ld16(tmem + lane_off + o_col, orr);
          ptx::tmem_ld_wait();
#pragma unroll
          for (int h = 0; h < G; ++h) o_acc[h] = __uint_as_float(orr[h]);
        } else {
          report_status(p.status, kStatusMmaTimeout);
        }
      }
      if (ti.nblk > 0) {  // the MMA warp counts only tasks with blocks
        ptx::tc_fence_before();
        ptx::mbar_arrive(&sh.o_free[ot]);
      }
      blk += ti.nblk;
      if (tr != nullptr && j == 1 && t == 0) tr[5] = ptx::globaltimer_ns();
      // output: thread t owns head-dimension row d = t
      const int hq0 = ti.kvh * G;
      if (ti.part < 0) {
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float v = l_run[h] > 0.f ? o_acc[h] / l_run[h] : 0.f;
          p.out[((size_t)ti.req * p.Hq + hq0 + h) * D + t] = __float2bfloat16(v);
        }
      } else {
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float v = l_run[h] > 0.f ? o_acc[h] / l_run[h] : 0.f;
          p.part_o[((size_t)ti.part * p.Hq + hq0 + h) * D + t] = v;
          if (t == 0)
            p.part_lse[(size_t)ti.part * p.Hq + hq0 + h] =
                l_run[h] > 0.f ? m_run[h] + __log2f(l_run[h]) : -INFINITY;
        }
        if (p.merge_cnt != nullptr) {
          // the last chunk of (request, KV head) to finish merges all chunks
          __threadfence();
          named_bar(1, kSoftmaxThreads);
          if (t == 0) {
            const uint32_t prev = atomicAdd(&p.merge_cnt[ti.req * p.Hkv + ti.kvh], 1u);
            sh.merge_last = prev == (uint32_t)(p.splits - 1);
          }
          named_bar(1, kSoftmaxThreads);
          if (sh.merge_last) {
            __threadfence();
            const int part0 = ti.req * p.splits;
            constexpr int SMAX = 8;  // the engine splits a request at most 8 ways
            bool merged = false;
            if constexpr (G * SMAX <= 32) {
              if (p.splits <= SMAX) {
                // every head's split LSEs and partial rows in ONE round of
                // independent L2 loads, ahead of any output store (per head,
                // the loads of head h+1 could not pass head h's store)
                float lse[G][SMAX], po[G][SMAX];
#pragma unroll
                for (int h = 0; h < G; ++h)
#pragma unroll
                  for (int s2 = 0; s2 < SMAX; ++s2) {
                    const bool in = s2 < p.splits;
                    lse[h][s2] = in ? __ldcg(&p.part_lse[(size_t)(part0 + s2) * p.Hq + hq0 + h]) : -INFINITY;
                    po[h][s2] = in ? __ldcg(&p.part_o[((size_t)(part0 + s2) * p.Hq + hq0 + h) * D + t]) : 0.f;
                  }
#pragma unroll
                for (int h = 0; h < G; ++h) {
                  float mx = -INFINITY, acc = 0.f, wsum = 0.f;
#pragma unroll
                  for (int s2 = 0; s2 < SMAX; ++s2)
                    if (s2 < p.splits) mx = fmaxf(mx, lse[h][s2]);
                  if (mx != -INFINITY) {
#pragma unroll
                    for (int s2 = 0; s2 < SMAX; ++s2) {  // fixed order: deterministic
                      if (s2 < p.splits) {
                        const float w = exp2f(lse[h][s2] - mx);
                        acc += w * po[h][s2];
                        wsum += w;
                      }
                    }
                  }
                  p.out[((size_t)ti.req * p.Hq + hq0 + h) * D + t] =
                      __float2bfloat16(wsum > 0.f ? acc / wsum : 0.f);
                }
                merged = true;
              }
            }
#pragma unroll
            for (int h = 0; h < G && !merged; ++h) {
              float mx = -INFINITY, acc = 0.f, wsum = 0.f;
              if (p.splits <= SMAX) {
                // every split's LSE and partial row of this head in one round of
                // independent loads (a loop over splits would wait for each)
                float lse[SMAX], po[SMAX];
#pragma unroll
                for (int s2 = 0; s2 < SMAX; ++s2) {
                  lse[s2] = s2 < p.splits ? __ldcg(&p.part_lse[(size_t)(part0 + s2) * p.Hq + hq0 + h]) : -INFINITY;
                  po[s2] = s2 < p.splits ? __ldcg(&p.part_o[((size_t)(part0 + s2) * p.Hq + hq0 + h) * D + t]) : 0.f;
                }
#pragma unroll
                for (int s2 = 0; s2 < SMAX; ++s2)
                  if (s2 < p.splits) mx = fmaxf(mx, lse[s2]);
                if (mx != -INFINITY) {
#pragma unroll
                  for (int s2 = 0; s2 < SMAX; ++s2) {  // fixed order: deterministic
                    if (s2 < p.splits) {
                      const float w = exp2f(lse[s2] - mx);
                      acc += w * po[s2];
                      wsum += w;
                    }
                  }
                }
              } else {
                for (int s2 = 0; s2 < p.splits; ++s2)
                  mx = fmaxf(mx, __ldcg(&p.part_lse[(size_t)(part0 + s2) * p.Hq + hq0 + h]));
                if (mx != -INFINITY) {
                  for (int s2 = 0; s2 < p.splits; ++s2) {  // fixed order: deterministic
                    const float w = exp2f(__ldcg(&p.part_lse[(size_t)(part0 + s2) * p.Hq + hq0 + h]) - mx);
                    acc += w * __ldcg(&p.part_o[((size_t)(part0 + s2) * p.Hq + hq0 + h) * D + t]);
                    wsum += w;
                  }
                }
              }
              p.out[((size_t)ti.req * p.Hq + hq0 + h) * D + t] =
                  __float2bfloat16(wsum > 0.f ? acc / wsum : 0.f);
            }
            if (t == 0) p.merge_cnt[ti.req * p.Hkv + ti.kvh] = 0u;
          }
          named_bar(1, kSoftmaxThreads);  // merge_last is rewritten by the next task
        }
      }
      if (WOVEN && t == 0) sched::timer_commit(sl, timer_off, (uint32_t)ti.task, t0);
      if (tr != nullptr && j == 1 && t == 0) tr[6] = ptx::globaltimer_ns();
      ptx::mbar_arrive(&sh.task_empty[slot]);
    }
  }

  __syncwarp();  // reconverge single-lane roles before the CTA barrier
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) ptx::tmem_dealloc(tmem, TMEM_COLS);
  if (tr != nullptr && threadIdx.x == 0) tr[7] = ptx::globaltimer_ns();
  if (WOVEN) {
    // ticket queue: the last worker to leave resets the counters for the next launch
    if (ACQ == (int)sched::Acquire::Ticket && dynamic && sl.queue != nullptr && threadIdx.x == 0) {
      __threadfence();
      const uint32_t done = atomicAdd(sl.queue + 1, 1u);
      if (done == gridDim.x - 1) {
        sl.queue[0] = 0u;
        sl.queue[1] = 0u;
        __threadfence();
      }
    }
  }
}

// Merge split-KV partials: out[b, hq, :] = sum_i w_i * o_i, w_i = 2^(lse_i - lse).
__global__ void merge_kernel(const float *part_o, const float *part_lse, const int32_t *merge_req,
                             const int32_t *merge_begin, int Hq, __nv_bfloat16 *out) {
  const int r = blockIdx.x;   // merge row (one split request)
  const int hq = blockIdx.y;  // query head
  const int d = threadIdx.x;  // 0..127
  const int b0 = merge_begin[r], b1 = merge_begin[r + 1];
  float mx = -INFINITY;
  for (int i = b0; i < b1; ++i) mx = fmaxf(mx, part_lse[(size_t)i * Hq + hq]);
  float acc = 0.f, wsum = 0.f;
  if (mx != -INFINITY) {
    for (int i = b0; i < b1; ++i) {
      const float w = exp2f(part_lse[(size_t)i * Hq + hq] - mx);
      acc += w * part_o[((size_t)i * Hq + hq) * D + d];
      wsum += w;
    }
  }
  out[((size_t)merge_req[r] * Hq + hq) * D + d] = __float2bfloat16(wsum > 0.f ? acc / wsum : 0.f);
}

template <int G, bool WOVEN, int ACQ>
static int launch(const CUtensorMap &tk, const CUtensorMap &tv, const CUtensorMap &tk2,
                  const CUtensorMap &tv2, const Params &p, int grid, cudaStream_t st) {
  auto kern = decode_kernel<G, WOVEN, ACQ>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    attr = true;
  }
  if (WOVEN) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kern, tk, tv, tk2, tv2, p);
  } else {
    kern<<<grid, kThreads, SMEM, st>>>(tk, tv, tk2, tv2, p);
  }
  return 0;
}

template <int G>
static int dispatch_acq(bool woven, int acq, const CUtensorMap &tk, const CUtensorMap &tv,
                        const CUtensorMap &tk2, const CUtensorMap &tv2, const Params &p, int grid,
                        cudaStream_t st) {
  if (!woven) return launch<G, false, 0>(tk, tv, tk2, tv2, p, grid, st);
  switch (acq) {
    case 1: return launch<G, true, 1>(tk, tv, tk2, tv2, p, grid, st);
    case 2: return launch<G, true, 2>(tk, tv, tk2, tv2, p, grid, st);
    default: return launch<G, true, 0>(tk, tv, tk2, tv2, p, grid, st);
  }
}

}  // namespace attn

extern "C" int sched_attn_decode_smem_bytes() { return attn::SMEM; }

// Resident CTAs per SM of the woven static kernel (the CLC prefix R = this x SMs).
// Diagnostic: when set, every decode-attention launch records its per-CTA
// phase trace here ([grid][8] u64, see Params::trace).
static unsigned long long *g_attn_trace = nullptr;
extern "C" void sched_attn_decode_set_trace(unsigned long long *trace) { g_attn_trace = trace; }

extern "C" int sched_attn_decode_occupancy(int group) {
  int blocks = 0;
  const void *k = nullptr;
  switch (group) {
    case 1: k = (const void *)attn::decode_kernel<1, true, 2>; break;
    case 2: k = (const void *)attn::decode_kernel<2, true, 2>; break;
    case 8: k = (const void *)attn::decode_kernel<8, true, 2>; break;
    default: k = (const void *)attn::decode_kernel<4, true, 2>; break;
  }
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, attn::SMEM);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, k, attn::kThreads, attn::SMEM) !=
      cudaSuccess)
    return 0;
  return blocks;
}

// q [B, Hq, 128] bf16; k_cache/v_cache [pages, Hkv, 16, 128] bf16;
// items [num_items] (req, kv_begin, kv_end, part); grid: tasks (static/CLC)
// or workers (ticket); a static launch with fewer CTAs than tasks strides.
// With merge_cnt, split requests (part >= 0, part = req * splits + s) are
// merged in-kernel by the last chunk to finish. Returns 0 on success.
extern "C" int sched_attn_decode(const void *q, void *out, const void *k_cache,
                                 const void *v_cache, int num_pages, const int32_t *block_table,
                                 int bt_stride, const void *items, int num_items, int Hq, int Hkv,
                                 float sm_scale, float *part_o, float *part_lse,
                                 uint32_t *merge_cnt, int splits, SchedSlots slots, int woven,
                                 int acquire, int grid, int pf_blocks, float dT, float dR, float H,
                                 const void *stage_k, const void *stage_v, int stage_pages,
                                 int stage_split, const void *l2_prefetch, long long l2_prefetch_bytes,
                                 int *status, cudaStream_t st) {
  if (num_items <= 0) return 0;
  if (stage_k != nullptr && (stage_v == nullptr || stage_pages <= 0 || stage_split <= 0)) return -1;
  const int G = Hq / Hkv;
  if (Hq % Hkv != 0 || (G != 1 && G != 2 && G != 4 && G != 8)) return -1;
  attn::Params p;
  p.q = static_cast<const __nv_bfloat16 *>(q);
  p.out = static_cast<__nv_bfloat16 *>(out);
  p.block_table = block_table;
  p.bt_stride = bt_stride;
  p.items = static_cast<const attn::Item *>(items);
  p.num_items = num_items;
  p.num_tasks = num_items * Hkv;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.part_o = part_o;
  p.part_lse = part_lse;
  p.merge_cnt = merge_cnt;
  p.splits = splits > 0 ? splits : 1;
  p.total_rows = num_pages * Hkv * attn::PS;
  p.stage_split = stage_k != nullptr ? stage_split : 0x7fffffff;
  p.num_pages = num_pages;
  p.stage_pages = stage_k != nullptr ? stage_pages : 0;
  p.slots = slots;
  p.pc.dT = dT;
  p.pc.dR = dR;
  p.pc.H = H;
  p.pf_blocks = pf_blocks;
  p.status = status;
  p.trace = g_attn_trace;
  p.l2_prefetch = (l2_prefetch != nullptr && (reinterpret_cast<uintptr_t>(l2_prefetch) & 15u) == 0 &&
                   l2_prefetch_bytes >= 16)
                      ? static_cast<const uint8_t *>(l2_prefetch)
                      : nullptr;
  p.l2_prefetch_bytes = l2_prefetch_bytes;
  if (grid <= 0) grid = p.num_tasks;
  try {
    const uint64_t rows = (uint64_t)num_pages * Hkv * attn::PS;
    CUtensorMap tk = tmap::make_kv_pages(k_cache, rows);
    CUtensorMap tv = tmap::make_kv_pages(v_cache, rows);
    CUtensorMap tk2 = tk, tv2 = tv;
    if (stage_k != nullptr) {
      const uint64_t srows = (uint64_t)stage_pages * Hkv * attn::PS;
      tk2 = tmap::make_kv_pages(stage_k, srows);
      tv2 = tmap::make_kv_pages(stage_v, srows);
    }
    switch (G) {
      case 1: attn::dispatch_acq<1>(woven, acquire, tk, tv, tk2, tv2, p, grid, st); break;
      case 2: attn::dispatch_acq<2>(woven, acquire, tk, tv, tk2, tv2, p, grid, st); break;
      case 8: attn::dispatch_acq<8>(woven, acquire, tk, tv, tk2, tv2, p, grid, st); break;
      default: attn::dispatch_acq<4>(woven, acquire, tk, tv, tk2, tv2, p, grid, st); break;
    }
  } catch (const std::exception &) {
    return -3;
  }
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int sched_attn_merge(const float *part_o, const float *part_lse,
                                const int32_t *merge_req, const int32_t *merge_begin, int rows,
                                int Hq, void *out, cudaStream_t st) {
  if (rows <= 0) return 0;
  attn::merge_kernel<<<dim3(rows, Hq), attn::D, 0, st>>>(
      part_o, part_lse, merge_req, merge_begin, Hq, static_cast<__nv_bfloat16 *>(out));
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}
