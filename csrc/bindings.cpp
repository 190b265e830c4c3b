// bindings.cpp -- torch-facing wrappers of the extern "C" launchers.
//
// Every op runs on the caller's current CUDA stream (so CUDA-graph capture
// and stream scoping compose with torch), checks devices, dtypes, shapes and
// alignment, and raises on a launcher error instead of returning silently.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdint>

#include "gemm_api.h"
#include "sched/abi.h"
#include "sp_api.h"

extern "C" {
int sched_attn_decode(const void *q, void *out, const void *k_cache, const void *v_cache,
                      int num_pages, const int32_t *block_table, int bt_stride, const void *items,
                      int num_items, int Hq, int Hkv, float sm_scale, float *part_o,
                      float *part_lse, uint32_t *merge_cnt, int splits, SchedSlots slots,
                      int woven, int acquire, int grid, int pf_blocks, float dT, float dR,
                      float H, const void *stage_k, const void *stage_v, int stage_pages,
                      int stage_split, const void *l2_prefetch, long long l2_prefetch_bytes, int *status,
                      cudaStream_t st);
int sched_attn_merge(const float *part_o, const float *part_lse, const int32_t *merge_req,
                     const int32_t *merge_begin, int rows, int Hq, void *out, cudaStream_t st);
int sched_attn_decode_occupancy(int group);
int sched_attn_decode_smem_bytes();
int sched_attn_prefill(const void *q, int q_rows, void *out, const void *k_cache, const void *v_cache,
                       int num_pages, const int32_t *block_table, int bt_stride,
                       const int32_t *kv_lens, const void *tiles, int num_tiles, int Hq, int Hkv,
                       int page_size, float sm_scale, int *status, cudaStream_t st);
int sched_attn_prefill_tile_rows();
int sched_add_rmsnorm(const void *x, void *res, const void *w, void *y, int T, int H, float eps,
                      cudaStream_t st);
int sched_rope_kv_append(const void *qkv, const int32_t *pos, const int32_t *slot,
                         const float *cos_sin, void *q_out, void *k_cache, void *v_cache, int T,
                         int Hq, int Hkv, int D, int page_size, int num_pages, int *status, cudaStream_t st);
int sched_embedding(const int32_t *ids, const int32_t *prev, int n_prev, const void *table, void *out, int T, int H,
                    int vocab, int *status, cudaStream_t st);
int sched_argmax(const void *logits, int T, int V, int ld, int32_t *ids, float *maxv,
                 int id_offset, cudaStream_t st);
int sched_moe_router(const void *x, const void *wr, int T, int H, int E, int K, int32_t *ids,
                     float *wts, cudaStream_t st);
int sched_moe_quantize(const void *in, int R, int I, void *out, float *scale,
                       const uint32_t *rows_valid, int rows_per_expert, cudaStream_t st);
int sched_moe_combine_norm(const void *c, int K, void *h, const void *w, void *y, int T, int H,
                           float eps, uint32_t *cnt, uint32_t *dropped_step, uint32_t *arrivals,
                           int *status, cudaStream_t st);
}
#include "moe_api.h"
extern "C" int sched_probe_stream(const void *src, size_t bytes, int policy, unsigned *sink, int grid,
                                  cudaStream_t st);
extern "C" int sched_probe_tasks(const uint32_t *cost, int n_tasks, int mode, int grid, int memory,
                                 const void *data, size_t data_bytes, unsigned *hits, unsigned *per_cta,
                                 unsigned *ticket, unsigned *sink, int *status, cudaStream_t st);
extern "C" int sched_probe_tasks_occupancy();
extern "C" void sched_attn_decode_set_trace(unsigned long long *trace);
extern "C" int sched_argmax_exchange(const void *logits, int T, int V, int ld, int32_t *ids, float *maxv,
                                     int id_offset, void *const *lines, int world, int rank, uint32_t *state,
                                     long long set_lines, int *status, cudaStream_t st);
extern "C" int sched_probe_clc_shape(const uint32_t *work, int gx, int gy, int gz, int stride, int cx,
                                     unsigned *hits, unsigned *claimed, unsigned *launched, unsigned *fails,
                                     unsigned *w_nonzero, int *status, cudaStream_t st);
extern "C" int sched_probe_clc_shape_capacity(int cx);
extern "C" int sched_probe_clc(const uint32_t *work, int n_tasks, int mode, int grid, int max_rec, unsigned *hits,
                               unsigned long long *rec, unsigned *n_rec, unsigned *smid, int *status,
                               cudaStream_t st);
extern "C" int sched_probe_mix(const void *R, size_t r_bytes, const void *S, size_t s_bytes, int mode, float frac,
                               unsigned *sink, int grid, cudaStream_t st);
extern "C" int sched_probe_pdl_pairs(float *buf, float *out, int n, const float *table, int work, int prologue,
                                     int pdl, int pairs, cudaStream_t st);
extern "C" int sched_probe_pdl_produce(float *buf, int n, int work, cudaStream_t st);
extern "C" int sched_kv_page_copy(const void *src_k, const void *src_v, long long src_pages, void *dst_k,
                                  void *dst_v, long long dst_pages, const int32_t *pairs, int n_pairs,
                                  const int *n_dev, int layers, int heads, int *status, cudaStream_t st);
extern "C" int sched_kv_page_copy_fp8(const void *src_k, const void *src_v, long long src_pages, void *dst_k,
                                      void *dst_v, long long dst_pages, float *scale_k, float *scale_v, int to_fp8,
                                      const int32_t *pairs, int n_pairs, const int *n_dev, int layers, int heads,
                                      int *status, cudaStream_t st);

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda(const at::Tensor &t, const char *name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
void check_bf16(const at::Tensor &t, const char *name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
}
void check_i32(const at::Tensor &t, const char *name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == at::kInt, name, " must be int32");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}
// A launcher's non-zero return code is recorded here instead of thrown:
// throwing a c10::Error out of a binding after its CUDA device guard has
// run crashed the process (SIGSEGV) on the B200 boxes, while throws before
// the guard (argument checks) are translated normally. The Python wrapper
// of every launcher (_ext._Counted) calls take_error() after the call and
// raises there.
namespace {
thread_local int g_last_rc = 0;
thread_local const char *g_last_op = "";
}  // namespace
void check_rc(int rc, const char *op) {
  if (rc != 0 && g_last_rc == 0) {
    g_last_rc = rc;
    g_last_op = op;
  }
}
std::tuple<int64_t, std::string> take_error() {
  std::tuple<int64_t, std::string> r{g_last_rc, std::string(g_last_op)};
  g_last_rc = 0;
  g_last_op = "";
  return r;
}

template <typename T>
T *ptr_or_null(const c10::optional<at::Tensor> &t) {
  return (t.has_value() && t->defined()) ? static_cast<T *>(t->data_ptr()) : nullptr;
}

// ---------------------------------------------------------------- GEMM
int num_sms(const at::Tensor &t) {
  static int n[64] = {0};
  const int d = t.get_device();
  if (d >= 0 && d < 64) {
    if (n[d] == 0) n[d] = at::cuda::getDeviceProperties(d)->multiProcessorCount;
    return n[d];
  }
  return 148;
}

// Diagnostic: when set, every GEMM launch records per-CTA timestamps here.
unsigned long long *g_gemm_trace = nullptr;
void set_attn_trace(int64_t ptr) { sched_attn_decode_set_trace(reinterpret_cast<unsigned long long *>(ptr)); }
void set_gemm_trace(int64_t ptr) { g_gemm_trace = reinterpret_cast<unsigned long long *>(ptr); }

// Residual add + RMSNorm fused after the projection: res += y, out = rmsnorm(res) * nw
// (all [T, N] bf16 except nw [N]); row_cnt int32 [>= T], zero between calls.
void set_norm(GemmArgs &a, const c10::optional<at::Tensor> &res, const c10::optional<at::Tensor> &nw,
              const c10::optional<at::Tensor> &out, const c10::optional<at::Tensor> &row_cnt, double eps) {
  if (!(nw.has_value() && nw->defined())) return;
  TORCH_CHECK(res.has_value() && out.has_value() && row_cnt.has_value(), "fused norm needs res, out and row_cnt");
  check_bf16(*res, "norm res");
  check_bf16(*nw, "norm weight");
  check_bf16(*out, "norm out");
  check_i32(*row_cnt, "row_cnt");
  TORCH_CHECK(res->is_contiguous() && out->is_contiguous() && nw->is_contiguous(), "contiguous norm tensors");
  TORCH_CHECK(res->dim() == 2 && res->size(0) >= a.T && res->size(1) == a.N && out->sizes() == res->sizes() &&
                  nw->numel() == a.N && row_cnt->numel() >= a.T,
              "norm tensors: res/out [>= T, N], weight [N], row_cnt [>= T]");
  a.norm_res = reinterpret_cast<__nv_bfloat16 *>(res->data_ptr());
  a.norm_w = reinterpret_cast<const __nv_bfloat16 *>(nw->data_ptr());
  a.norm_out = reinterpret_cast<__nv_bfloat16 *>(out->data_ptr());
  a.row_cnt = reinterpret_cast<uint32_t *>(row_cnt->data_ptr<int32_t>());
  a.norm_eps = (float)eps;
}

GemmArgs base_args(const at::Tensor &x, const at::Tensor &w, int64_t grid,
                   const c10::optional<at::Tensor> &ws, const c10::optional<at::Tensor> &counters,
                   const c10::optional<at::Tensor> &status) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2, "gemm expects 2-D operands");
  TORCH_CHECK(x.stride(1) == 1 && w.is_contiguous(), "row-major operands");
  TORCH_CHECK(w.size(1) == x.size(1), "K mismatch");
  GemmArgs a{};
  a.x = x.data_ptr();
  a.ldx = x.stride(0);
  a.w = w.data_ptr();
  a.T = x.size(0);
  a.K = x.size(1);
  a.N = w.size(0);
  a.grid = grid;
  a.num_sms = num_sms(x);
  a.trace = g_gemm_trace;
  a.ws = ptr_or_null<float>(ws);
  a.ws_floats = (ws.has_value() && ws->defined()) ? ws->numel() : 0;
  a.counters = ptr_or_null<uint32_t>(counters);
  a.counter_count = (counters.has_value() && counters->defined()) ? counters->numel() : 0;
  a.status = ptr_or_null<int>(status);
  return a;
}

// x_ready: address of the gathered rows' ready flags (0: x is local and ready)
void gemm(const at::Tensor &x, const at::Tensor &w, at::Tensor &y, int64_t epi, int64_t grid,
          const c10::optional<at::Tensor> &ws, const c10::optional<at::Tensor> &counters,
          const c10::optional<at::Tensor> &status, int64_t x_ready, const c10::optional<at::Tensor> &norm_res,
          const c10::optional<at::Tensor> &norm_w, const c10::optional<at::Tensor> &norm_out,
          const c10::optional<at::Tensor> &row_cnt, double norm_eps) {
  GemmArgs a = base_args(x, w, grid, ws, counters, status);
  a.x_ready = reinterpret_cast<const uint32_t *>(x_ready);
  check_bf16(y, "y");
  TORCH_CHECK(y.dim() == 2 && y.stride(1) == 1 && y.size(0) >= a.T, "y [T, ldy]");
  TORCH_CHECK(epi == kEpiStore ? y.size(1) >= a.N : y.size(1) >= a.N / 2, "y columns");
  TORCH_CHECK(epi == kEpiStore || epi == kEpiSwiGLU, "use gemm_qkv_rope for the QKV epilogue");
  a.y = y.data_ptr();
  a.ldy = y.stride(0);
  a.epi = epi;
  TORCH_CHECK(!(norm_w.has_value() && norm_w->defined()) || epi == kEpiStore, "the fused norm follows a plain store");
  set_norm(a, norm_res, norm_w, norm_out, row_cnt, norm_eps);
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(x.device());
    rc_ = sched_gemm_run(&a, cur_stream());
  }
  check_rc(rc_, "gemm");
}

void gemm_qkv_rope(const at::Tensor &x, const at::Tensor &w, const at::Tensor &pos,
                   const at::Tensor &slot, const at::Tensor &cos_sin, at::Tensor &q_out,
                   at::Tensor &k_cache, at::Tensor &v_cache, int64_t Hq, int64_t Hkv,
                   int64_t grid, const c10::optional<at::Tensor> &ws,
                   const c10::optional<at::Tensor> &counters,
                   const c10::optional<at::Tensor> &status, int64_t x_ready) {
  GemmArgs a = base_args(x, w, grid, ws, counters, status);
  a.x_ready = reinterpret_cast<const uint32_t *>(x_ready);
  check_i32(pos, "pos");
  check_i32(slot, "slot");
  check_bf16(q_out, "q_out");
  check_bf16(k_cache, "k_cache");
  check_bf16(v_cache, "v_cache");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous(), "cos_sin float32");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(3) == 128 && k_cache.is_contiguous(), "cache layout");
  TORCH_CHECK(q_out.is_contiguous() && q_out.numel() >= a.T * Hq * 128, "q_out [T, Hq, 128]");
  a.epi = kEpiRopeKV;
  a.pos = pos.data_ptr<int32_t>();
  a.slot = slot.data_ptr<int32_t>();
  a.cos_sin = cos_sin.data_ptr<float>();
  a.q_out = reinterpret_cast<__nv_bfloat16 *>(q_out.data_ptr());
  a.k_cache = reinterpret_cast<__nv_bfloat16 *>(k_cache.data_ptr());
  a.v_cache = reinterpret_cast<__nv_bfloat16 *>(v_cache.data_ptr());
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.page_size = k_cache.size(2);
  a.kv_pages = k_cache.size(0);
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(x.device());
    rc_ = sched_gemm_run(&a, cur_stream());
  }
  check_rc(rc_, "gemm_qkv_rope");
}

// Row-parallel projection with the all-reduce fused into the GEMM epilogue.
// recv/flags: this process's addresses of every rank's slab and flag array.
// ll_state (int32 [2] on this device) selects the low-latency exchange:
// recv then holds every rank's line buffer (two sets of ll_set_lines
// 16-byte lines) and flags is ignored.
void gemm_allreduce(const at::Tensor &x, const at::Tensor &w, at::Tensor &y, int64_t rank,
                    int64_t world, const std::vector<int64_t> &recv,
                    const std::vector<int64_t> &flags, int64_t grid,
                    const c10::optional<at::Tensor> &ws,
                    const c10::optional<at::Tensor> &counters,
                    const c10::optional<at::Tensor> &status,
                    const c10::optional<at::Tensor> &ll_state, int64_t ll_set_lines,
                    const c10::optional<at::Tensor> &norm_res, const c10::optional<at::Tensor> &norm_w,
                    const c10::optional<at::Tensor> &norm_out, const c10::optional<at::Tensor> &row_cnt,
                    double norm_eps, int64_t ll_mc) {
  GemmArgs a = base_args(x, w, grid, ws, counters, status);
  check_bf16(y, "y");
  TORCH_CHECK(y.dim() == 2 && y.stride(1) == 1 && y.size(1) >= a.N, "y [T, >= N]");
  const bool ll = ll_state.has_value() && ll_state->defined();
  TORCH_CHECK(world >= 1 && world <= kMaxWorld && (int64_t)recv.size() == world &&
                  (ll || (int64_t)flags.size() == world),
              "one slab and one flag array per rank");
  if (ll) {
    check_i32(*ll_state, "ll_state");
    TORCH_CHECK(ll_state->numel() >= 2 && ll_state->device() == x.device(), "ll_state: int32 [2] on x's device");
    TORCH_CHECK(ll_set_lines >= world * a.T * (a.N / 4), "line buffer too small for [world, T, N/4] lines");
  }
  a.y = y.data_ptr();
  a.ldy = y.stride(0);
  a.epi = kEpiAllReduce;
  a.rank = rank;
  a.world = world;
  for (int j = 0; j < world; ++j) {
    a.recv[j] = reinterpret_cast<__nv_bfloat16 *>(recv[j]);
    a.flags[j] = ll ? nullptr : reinterpret_cast<uint32_t *>(flags[j]);
  }
  if (ll) {
    a.ll_state = reinterpret_cast<uint32_t *>(ll_state->data_ptr<int32_t>());
    a.ll_set_lines = ll_set_lines;
    a.ll_mc = reinterpret_cast<void *>(ll_mc);
  }
  set_norm(a, norm_res, norm_w, norm_out, row_cnt, norm_eps);
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(x.device());
    rc_ = sched_gemm_run(&a, cur_stream());
  }
  check_rc(rc_, "gemm_allreduce");
}

// Row-parallel projection, sequence-parallel output: each finished row goes
// to the slab of the rank that owns the token (kEpiReduceScatter); the owner
// reduces it in sp_reduce_norm. recv/flags: every rank's slab and row flags.
void gemm_reduce_scatter(const at::Tensor &x, const at::Tensor &w, int64_t rank, int64_t world,
                         const std::vector<int64_t> &recv, const std::vector<int64_t> &flags,
                         int64_t grid, const c10::optional<at::Tensor> &ws,
                         const c10::optional<at::Tensor> &counters,
                         const c10::optional<at::Tensor> &status) {
  GemmArgs a = base_args(x, w, grid, ws, counters, status);
  TORCH_CHECK(world >= 1 && world <= kMaxWorld && (int64_t)recv.size() == world &&
                  (int64_t)flags.size() == world,
              "one slab and one flag array per rank");
  a.epi = kEpiReduceScatter;
  a.rank = rank;
  a.world = world;
  for (int j = 0; j < world; ++j) {
    a.recv[j] = reinterpret_cast<__nv_bfloat16 *>(recv[j]);
    a.flags[j] = reinterpret_cast<uint32_t *>(flags[j]);
  }
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(x.device());
    rc_ = sched_gemm_run(&a, cur_stream());
  }
  check_rc(rc_, "gemm_reduce_scatter");
}

// Sequence-parallel reduce + residual + RMSNorm + all-gather push (sp_api.h).
void sp_reduce_norm(int64_t slab, int64_t row_flags, at::Tensor &res, const at::Tensor &w,
                    const c10::optional<at::Tensor> &delta, const std::vector<int64_t> &gather,
                    const std::vector<int64_t> &ready, int64_t clear, int64_t clear_n, int64_t T,
                    int64_t rank, int64_t world, double eps, const c10::optional<at::Tensor> &status) {
  check_bf16(res, "res");
  check_bf16(w, "w");
  TORCH_CHECK(res.dim() == 2 && res.is_contiguous() && res.size(0) >= T, "res [>= T, H] contiguous");
  const int64_t H = res.size(1);
  TORCH_CHECK(w.numel() == H && w.is_contiguous(), "w [H]");
  TORCH_CHECK(world >= 1 && world <= kMaxWorld && (int64_t)gather.size() == world &&
                  (int64_t)ready.size() == world && rank >= 0 && rank < world,
              "one gather buffer and one ready array per rank");
  SpNormArgs a{};
  a.slab = reinterpret_cast<const __nv_bfloat16 *>(slab);
  a.row_flags = reinterpret_cast<uint32_t *>(row_flags);
  a.res = reinterpret_cast<__nv_bfloat16 *>(res.data_ptr());
  a.w = reinterpret_cast<const __nv_bfloat16 *>(w.data_ptr());
  if (delta.has_value() && delta->defined()) {
    check_bf16(*delta, "delta");
    TORCH_CHECK(delta->is_contiguous() && delta->size(0) >= T && delta->size(1) == H, "delta [>= T, H]");
    a.delta = reinterpret_cast<__nv_bfloat16 *>(delta->data_ptr());
  }
  for (int j = 0; j < world; ++j) {
    a.gather[j] = reinterpret_cast<__nv_bfloat16 *>(gather[j]);
    a.ready[j] = reinterpret_cast<uint32_t *>(ready[j]);
  }
  a.clear = reinterpret_cast<uint32_t *>(clear);
  a.clear_n = clear_n;
  a.T = T;
  a.H = H;
  a.rank = rank;
  a.world = world;
  a.eps = (float)eps;
  a.status = ptr_or_null<int>(status);
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(res.device());
    rc_ = sched_sp_reduce_norm(&a, cur_stream());
  }
  check_rc(rc_, "sp_reduce_norm");
}

void sp_wait_rows(int64_t ready, int64_t T, const at::Tensor &status) {
  check_cuda(status, "status");
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(status.device());
    rc_ = sched_sp_wait_rows(reinterpret_cast<const uint32_t *>(ready), T,
                                static_cast<int *>(status.data_ptr()), cur_stream());
  }
  check_rc(rc_, "sp_wait_rows");
}

int64_t gemm_ws_floats(int64_t T, int64_t N, int64_t K, int64_t grid) {
  return sched_gemm_ws_floats(T, N, K, grid);
}

// ---------------------------------------------------------------- attention
SchedSlots make_slots(const c10::optional<at::Tensor> &order, const c10::optional<at::Tensor> &ctrl,
                      const c10::optional<at::Tensor> &timer, const c10::optional<at::Tensor> &queue,
                      int64_t max_tasks) {
  SchedSlots s{};
  s.order = ptr_or_null<const int32_t>(order);
  s.ctrl = ptr_or_null<const SchedCtrl>(ctrl);
  s.timer = ptr_or_null<unsigned long long>(timer);
  s.queue = ptr_or_null<uint32_t>(queue);
  s.max_tasks = static_cast<uint32_t>(max_tasks);
  return s;
}

void attn_decode(const at::Tensor &q, at::Tensor &out, const at::Tensor &k_cache,
                 const at::Tensor &v_cache, const at::Tensor &block_table, const at::Tensor &items,
                 int64_t num_items, double sm_scale, const c10::optional<at::Tensor> &part_o,
                 const c10::optional<at::Tensor> &part_lse,
                 const c10::optional<at::Tensor> &merge_cnt, int64_t splits,
                 const c10::optional<at::Tensor> &order, const c10::optional<at::Tensor> &ctrl,
                 const c10::optional<at::Tensor> &timer, const c10::optional<at::Tensor> &queue,
                 int64_t max_tasks, int64_t woven, int64_t acquire, int64_t grid,
                 int64_t pf_blocks, double dT, double dR, double H,
                 const c10::optional<at::Tensor> &stage_k, const c10::optional<at::Tensor> &stage_v,
                 int64_t stage_split, const c10::optional<at::Tensor> &status, int64_t l2_prefetch,
                 int64_t l2_prefetch_bytes) {
  check_bf16(q, "q");
  check_bf16(out, "out");
  check_bf16(k_cache, "k_cache");
  const bool staged = stage_k.has_value() && stage_k->defined();
  if (staged) {
    TORCH_CHECK(stage_v.has_value() && stage_v->defined() && stage_k->is_contiguous() && stage_v->is_contiguous() &&
                    stage_k->dim() == 4 && stage_k->size(1) == k_cache.size(1),
                "staging pool [pages, Hkv, 16, 128]");
  }
  check_bf16(v_cache, "v_cache");
  check_i32(block_table, "block_table");
  check_i32(items, "items");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && q.is_contiguous(), "q [B, Hq, 128]");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(2) == 16 && k_cache.size(3) == 128 &&
                  k_cache.is_contiguous() && v_cache.sizes() == k_cache.sizes(),
              "cache [pages, Hkv, 16, 128]");
  TORCH_CHECK(items.numel() >= num_items * 4, "items [n, 4]");
  const int Hq = q.size(1), Hkv = k_cache.size(1);
  TORCH_CHECK(Hkv > 0 && Hq % Hkv == 0 && (Hq / Hkv == 1 || Hq / Hkv == 2 || Hq / Hkv == 4 || Hq / Hkv == 8),
              "query heads per KV head must be 1, 2, 4 or 8");
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(q.device());
    SchedSlots sl = make_slots(order, ctrl, timer, queue, max_tasks);
    rc_ = sched_attn_decode(q.data_ptr(), out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                               k_cache.size(0), block_table.data_ptr<int32_t>(),
                               block_table.stride(0), items.data_ptr(), num_items, Hq, Hkv,
                               (float)sm_scale, ptr_or_null<float>(part_o),
                               ptr_or_null<float>(part_lse), ptr_or_null<uint32_t>(merge_cnt),
                               splits, sl, woven, acquire, grid, pf_blocks,
                               (float)dT, (float)dR, (float)H, staged ? stage_k->data_ptr() : nullptr,
                               staged ? stage_v->data_ptr() : nullptr, staged ? (int)stage_k->size(0) : 0,
                               (int)stage_split, reinterpret_cast<const void *>(l2_prefetch),
                               (long long)l2_prefetch_bytes, ptr_or_null<int>(status), cur_stream());
  }
  check_rc(rc_, "attn_decode");
}

void attn_merge(const at::Tensor &part_o, const at::Tensor &part_lse, const at::Tensor &merge_req,
                const at::Tensor &merge_begin, int64_t rows, at::Tensor &out) {
  check_i32(merge_req, "merge_req");
  check_i32(merge_begin, "merge_begin");
  check_bf16(out, "out");
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(out.device());
    rc_ = sched_attn_merge(part_o.data_ptr<float>(), part_lse.data_ptr<float>(),
                              merge_req.data_ptr<int32_t>(), merge_begin.data_ptr<int32_t>(), rows,
                              out.size(1), out.data_ptr(), cur_stream());
  }
  check_rc(rc_, "attn_merge");
}

void attn_prefill(const at::Tensor &q, at::Tensor &out, const at::Tensor &k_cache,
                  const at::Tensor &v_cache, const at::Tensor &block_table,
                  const at::Tensor &kv_lens, const at::Tensor &tiles, int64_t num_tiles,
                  double sm_scale, const c10::optional<at::Tensor> &status) {
  check_bf16(q, "q");
  check_bf16(out, "out");
  check_bf16(k_cache, "k_cache");
  check_bf16(v_cache, "v_cache");
  check_i32(block_table, "block_table");
  check_i32(kv_lens, "kv_lens");
  check_i32(tiles, "tiles");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && q.is_contiguous(), "q [T, Hq, 128]");
  TORCH_CHECK(out.sizes() == q.sizes() && out.is_contiguous(), "out like q");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(2) == 16 && k_cache.size(3) == 128 &&
                  k_cache.is_contiguous() && v_cache.sizes() == k_cache.sizes() && v_cache.is_contiguous(),
              "cache [pages, Hkv, 16, 128]");
  TORCH_CHECK(k_cache.size(1) > 0 && q.size(1) % k_cache.size(1) == 0, "query heads per KV head");
  TORCH_CHECK(tiles.numel() >= num_tiles * 4 && tiles.is_contiguous(), "tiles [n, 4]");
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(q.device());
    rc_ = sched_attn_prefill(q.data_ptr(), q.size(0), out.data_ptr(), k_cache.data_ptr(),
                             v_cache.data_ptr(), k_cache.size(0), block_table.data_ptr<int32_t>(), block_table.stride(0),
                             kv_lens.data_ptr<int32_t>(), tiles.data_ptr(), num_tiles, q.size(1),
                             k_cache.size(1), k_cache.size(2), (float)sm_scale,
                             ptr_or_null<int>(status), cur_stream());
  }
  check_rc(rc_, "attn_prefill");
}

int64_t attn_decode_occupancy(int64_t group) { return sched_attn_decode_occupancy(group); }
int64_t attn_decode_smem_bytes() { return sched_attn_decode_smem_bytes(); }

// ---------------------------------------------------------------- elementwise
void add_rmsnorm(const at::Tensor &x, const c10::optional<at::Tensor> &res, const at::Tensor &w,
                 at::Tensor &y, double eps) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_bf16(y, "y");
  TORCH_CHECK(x.is_contiguous() && y.is_contiguous(), "contiguous rows");
  const int H = x.size(-1), T = x.numel() / H;
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(x.device());
    rc_ = sched_add_rmsnorm(x.data_ptr(), res.has_value() ? res->data_ptr() : nullptr,
                               w.data_ptr(), y.data_ptr(), T, H, (float)eps, cur_stream());
  }
  check_rc(rc_, "add_rmsnorm");
}

void rope_kv_append(const at::Tensor &qkv, const at::Tensor &pos, const at::Tensor &slot,
                    const at::Tensor &cos_sin, at::Tensor &q_out, at::Tensor &k_cache,
                    at::Tensor &v_cache, int64_t Hq, int64_t Hkv, const c10::optional<at::Tensor> &status) {
  check_bf16(qkv, "qkv");
  check_i32(pos, "pos");
  check_i32(slot, "slot");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous(), "cos_sin float32");
  const int T = qkv.size(0);
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(qkv.device());
    rc_ = sched_rope_kv_append(qkv.data_ptr(), pos.data_ptr<int32_t>(), slot.data_ptr<int32_t>(),
                                  cos_sin.data_ptr<float>(), q_out.data_ptr(), k_cache.data_ptr(),
                                  v_cache.data_ptr(), T, Hq, Hkv, k_cache.size(3), k_cache.size(2),
                                  k_cache.size(0), ptr_or_null<int>(status), cur_stream());
  }
  check_rc(rc_, "rope_kv_append");
}

void embedding(const at::Tensor &ids, const at::Tensor &table, at::Tensor &out,
               const c10::optional<at::Tensor> &status, const c10::optional<at::Tensor> &prev) {
  check_i32(ids, "ids");
  check_bf16(table, "table");
  const bool has_prev = prev.has_value() && prev->defined();
  if (has_prev) check_i32(*prev, "prev");
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(ids.device());
    rc_ = sched_embedding(ids.data_ptr<int32_t>(), has_prev ? prev->data_ptr<int32_t>() : nullptr,
                             has_prev ? (int)prev->numel() : 0, table.data_ptr(), out.data_ptr(), ids.numel(),
                             table.size(1), table.size(0), ptr_or_null<int>(status), cur_stream());
  }
  check_rc(rc_, "embedding");
}

void argmax_exchange(const at::Tensor &logits, at::Tensor &ids, int64_t id_offset,
                     const std::vector<int64_t> &lines, int64_t rank, at::Tensor &state, int64_t set_lines,
                     const c10::optional<at::Tensor> &status) {
  check_bf16(logits, "logits");
  check_i32(ids, "ids");
  check_i32(state, "state");
  const int64_t world = (int64_t)lines.size();
  TORCH_CHECK(world >= 1 && world <= 8 && rank >= 0 && rank < world, "one line buffer per rank (<= 8)");
  TORCH_CHECK(state.numel() >= 2 && set_lines >= world * logits.size(0), "state [2]; set_lines >= world x rows");
  std::vector<void *> ptrs(world);
  for (int64_t j = 0; j < world; ++j) ptrs[j] = reinterpret_cast<void *>(lines[j]);
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(logits.device());
    rc_ = sched_argmax_exchange(logits.data_ptr(), logits.size(0), logits.size(1), logits.stride(0),
                                ids.data_ptr<int32_t>(), nullptr, id_offset, ptrs.data(), (int)world, (int)rank,
                                reinterpret_cast<uint32_t *>(state.data_ptr<int32_t>()), set_lines,
                                ptr_or_null<int>(status), cur_stream());
  }
  check_rc(rc_, "argmax_exchange");
}

void argmax(const at::Tensor &logits, at::Tensor &ids, const c10::optional<at::Tensor> &maxv,
            int64_t id_offset) {
  check_bf16(logits, "logits");
  check_i32(ids, "ids");
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(logits.device());
    rc_ = sched_argmax(logits.data_ptr(), logits.size(0), logits.size(1), logits.stride(0),
                          ids.data_ptr<int32_t>(), ptr_or_null<float>(maxv), id_offset, cur_stream());
  }
  check_rc(rc_, "argmax");
}

// ---------------------------------------------------------------- MoE
void moe_router(const at::Tensor &x, const at::Tensor &wr, at::Tensor &ids, at::Tensor &wts, int64_t k) {
  check_bf16(x, "x");
  check_bf16(wr, "wr");
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(x.device());
    rc_ = sched_moe_router(x.data_ptr(), wr.data_ptr(), x.size(0), x.size(1), wr.size(0), k,
                              ids.data_ptr<int32_t>(), wts.data_ptr<float>(), cur_stream());
  }
  check_rc(rc_, "moe_router");
}

// p: dict-like flat vector of int64 arguments (see sched_pass_b200/parallel/ep.py)
void moe_dispatch(const at::Tensor &x, const at::Tensor &ids, const at::Tensor &wts, int64_t T,
                  int64_t K, int64_t E, int64_t E_local, int64_t rank, int64_t world, int64_t capacity,
                  int64_t rows, const std::vector<int64_t> &slab, const std::vector<int64_t> &slab_scale,
                  const std::vector<int64_t> &slab_meta, const std::vector<int64_t> &counter,
                  const std::vector<int64_t> &done, int64_t local_done, int64_t combine_local,
                  int64_t dropped_step, int64_t dropped_total, const c10::optional<at::Tensor> &status) {
  moe::DispatchArgs a{};
  a.x = reinterpret_cast<const __nv_bfloat16 *>(x.data_ptr());
  a.ids = ids.data_ptr<int32_t>();
  a.wts = wts.data_ptr<float>();
  a.T = T;
  a.H = x.size(1);
  a.K = K;
  a.E = E;
  a.E_local = E_local;
  a.rank = rank;
  a.world = world;
  a.capacity = capacity;
  a.rows_per_expert = rows;
  for (int r = 0; r < world; ++r) {
    a.slab[r] = reinterpret_cast<uint8_t *>(slab[r]);
    a.slab_scale[r] = reinterpret_cast<float *>(slab_scale[r]);
    a.slab_meta[r] = reinterpret_cast<int32_t *>(slab_meta[r]);
    a.counter[r] = reinterpret_cast<uint32_t *>(counter[r]);
    a.done[r] = reinterpret_cast<uint32_t *>(done[r]);
  }
  a.local_done = reinterpret_cast<uint32_t *>(local_done);
  a.combine_local = reinterpret_cast<__nv_bfloat16 *>(combine_local);
  a.dropped_step = reinterpret_cast<uint32_t *>(dropped_step);
  a.dropped_total = reinterpret_cast<uint32_t *>(dropped_total);
  a.status = ptr_or_null<int>(status);
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(x.device());
    rc_ = sched_moe_dispatch(&a, cur_stream());
  }
  check_rc(rc_, "moe_dispatch");
}

void moe_expert_gemm(int64_t epi, const at::Tensor &w, int64_t x_ptr, int64_t E_local, int64_t N, int64_t K,
                     int64_t rows, const at::Tensor &w_scale, int64_t x_scale, int64_t act, int64_t counter,
                     int64_t done, int64_t rows_valid, int64_t tiles_done, int64_t world, int64_t capacity,
                     int64_t meta, const std::vector<int64_t> &combine, const std::vector<int64_t> &combine_cnt,
                     int64_t k_top, int64_t ws, int64_t tile_counters, int64_t grid, int64_t trace,
                     const c10::optional<at::Tensor> &status) {
  TORCH_CHECK(w.is_cuda() && w.element_size() == 1, "w: fp8 e4m3 [E_local * N, K]");
  moe::ExpertArgs a{};
  a.E_local = E_local;
  a.N = N;
  a.K = K;
  a.rows_per_expert = rows;
  a.w_scale = w_scale.data_ptr<float>();
  a.x_scale = reinterpret_cast<const float *>(x_scale);
  a.act = reinterpret_cast<__nv_bfloat16 *>(act);
  a.counter = reinterpret_cast<uint32_t *>(counter);
  a.done = reinterpret_cast<uint32_t *>(done);
  a.rows_valid = reinterpret_cast<uint32_t *>(rows_valid);
  a.tiles_done = reinterpret_cast<uint32_t *>(tiles_done);
  a.world = world;
  a.capacity = capacity;
  a.meta = reinterpret_cast<const int32_t *>(meta);
  for (size_t r = 0; r < combine.size() && r < moe::kMaxWorld; ++r) {
    a.combine[r] = reinterpret_cast<__nv_bfloat16 *>(combine[r]);
    a.combine_cnt[r] = reinterpret_cast<uint32_t *>(combine_cnt[r]);
  }
  a.k_top = k_top;
  a.ws = reinterpret_cast<float *>(ws);
  a.tile_counters = reinterpret_cast<uint32_t *>(tile_counters);
  a.grid = grid;
  a.trace = reinterpret_cast<unsigned long long *>(trace);
  a.status = ptr_or_null<int>(status);
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(w.device());
    rc_ = sched_moe_expert_gemm(epi, w.data_ptr(), reinterpret_cast<const void *>(x_ptr), &a, cur_stream());
  }
  check_rc(rc_, "moe_expert_gemm");
}

void moe_quantize(int64_t in, int64_t R, int64_t I, int64_t out, int64_t scale, int64_t rows_valid,
                  int64_t rows) {
  check_rc(sched_moe_quantize(reinterpret_cast<const void *>(in), R, I, reinterpret_cast<void *>(out),
                              reinterpret_cast<float *>(scale), reinterpret_cast<const uint32_t *>(rows_valid),
                              rows, cur_stream()),
           "moe_quantize");
}

void moe_combine_norm(int64_t c, int64_t K, at::Tensor &h, const at::Tensor &w, at::Tensor &y, int64_t T,
                      double eps, int64_t cnt, int64_t dropped_step, int64_t arrivals,
                      const c10::optional<at::Tensor> &status) {
  check_bf16(h, "h");
  check_bf16(y, "y");
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(h.device());
    rc_ = sched_moe_combine_norm(reinterpret_cast<const void *>(c), K, h.data_ptr(), w.data_ptr(), y.data_ptr(), T,
                                    h.size(1), (float)eps, reinterpret_cast<uint32_t *>(cnt),
                                    reinterpret_cast<uint32_t *>(dropped_step), reinterpret_cast<uint32_t *>(arrivals),
                                    ptr_or_null<int>(status), cur_stream());
  }
  check_rc(rc_, "moe_combine_norm");
}

void probe_stream(const at::Tensor &src, int64_t policy, at::Tensor &sink, int64_t grid) {
  TORCH_CHECK(src.is_cuda() && src.is_contiguous(), "src on the device");
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(src.device());
    rc_ = sched_probe_stream(src.data_ptr(), src.numel() * src.element_size(), policy,
                                reinterpret_cast<unsigned *>(sink.data_ptr()), grid, cur_stream());
  }
  check_rc(rc_, "probe_stream");
}

void probe_tasks(const at::Tensor &cost, int64_t mode, int64_t grid, int64_t memory, const at::Tensor &data,
                 at::Tensor &hits, at::Tensor &per_cta, at::Tensor &ticket, at::Tensor &sink,
                 const c10::optional<at::Tensor> &status) {
  TORCH_CHECK(cost.is_cuda() && cost.scalar_type() == at::kInt, "cost int32 on the device");
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(cost.device());
    rc_ = sched_probe_tasks(reinterpret_cast<const uint32_t *>(cost.data_ptr()), cost.numel(), mode, grid, memory,
                               data.data_ptr(), data.numel() * data.element_size(),
                               reinterpret_cast<unsigned *>(hits.data_ptr()),
                               reinterpret_cast<unsigned *>(per_cta.data_ptr()),
                               reinterpret_cast<unsigned *>(ticket.data_ptr()),
                               reinterpret_cast<unsigned *>(sink.data_ptr()), ptr_or_null<int>(status), cur_stream());
  }
  check_rc(rc_, "probe_tasks");
}

// counters: int32 [4n + 1] on the device: hits, claimed, launched, fails
// (n each) and the count of claim answers with a non-zero fourth word.
void probe_clc_shape(const at::Tensor &work, int64_t gx, int64_t gy, int64_t gz, int64_t stride, int64_t cx,
                     at::Tensor &counters, const c10::optional<at::Tensor> &status) {
  TORCH_CHECK(work.is_cuda() && work.scalar_type() == at::kInt && work.is_contiguous(), "work int32 on the device");
  TORCH_CHECK(gx > 0 && gy > 0 && gz > 0 && stride > 0 && cx >= 1 && cx <= 8 && gx % cx == 0,
              "grid dims > 0, stride > 0, cluster 1..8 dividing gx");
  const int64_t n = gx * gy * gz;
  TORCH_CHECK(work.numel() >= n, "work: one entry per CTA");
  TORCH_CHECK(counters.is_cuda() && counters.element_size() == 4 && counters.is_contiguous() &&
                  counters.numel() >= 4 * n + 1,
              "counters: int32 [4 n + 1]");
  unsigned *c = reinterpret_cast<unsigned *>(counters.data_ptr());
  int rc_ = 0;
  {  // the guard is gone before the launch code is recorded
    c10::cuda::CUDAGuard gd(work.device());
    rc_ = sched_probe_clc_shape(reinterpret_cast<const uint32_t *>(work.data_ptr()), (int)gx, (int)gy, (int)gz,
                                (int)stride, (int)cx, c, c + n, c + 2 * n, c + 3 * n, c + 4 * n,
                                ptr_or_null<int>(status), cur_stream());
  }
  check_rc(rc_, "probe_clc_shape");
}

void probe_clc(const at::Tensor &work, int64_t mode, int64_t grid, at::Tensor &hits, at::Tensor &rec,
               at::Tensor &n_rec, at::Tensor &smid, const c10::optional<at::Tensor> &status) {
  TORCH_CHECK(work.is_cuda() && work.scalar_type() == at::kInt && work.is_contiguous(), "work int32 on the device");
  TORCH_CHECK(mode >= 0 && mode <= 2, "mode is 0 (static), 1 (CLC late bound) or 2 (CLC claim-ahead)");
  const int64_t n = work.numel();
  const int64_t g = mode == 0 ? grid : n;
  TORCH_CHECK(g > 0, "grid must be positive");
  TORCH_CHECK(hits.numel() >= n && hits.element_size() == 4, "hits: int32 [n_tasks]");
  TORCH_CHECK(rec.dim() == 2 && rec.size(0) >= g && rec.element_size() == 8 && rec.is_contiguous(),
              "rec: int64 [grid, max_rec]");
  TORCH_CHECK(n_rec.numel() >= g && smid.numel() >= g && n_rec.element_size() == 4 && smid.element_size() == 4,
              "n_rec, smid: int32 [grid]");
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard gd(work.device());
    rc_ = sched_probe_clc(reinterpret_cast<const uint32_t *>(work.data_ptr()), (int)n, (int)mode, (int)g,
                             (int)rec.size(1), reinterpret_cast<unsigned *>(hits.data_ptr()),
                             reinterpret_cast<unsigned long long *>(rec.data_ptr()),
                             reinterpret_cast<unsigned *>(n_rec.data_ptr()), reinterpret_cast<unsigned *>(smid.data_ptr()),
                             ptr_or_null<int>(status), cur_stream());
  }
  check_rc(rc_, "probe_clc");
}

void probe_mix(const at::Tensor &R, const at::Tensor &S, int64_t mode, double frac, at::Tensor &sink,
               int64_t grid) {
  TORCH_CHECK(R.is_cuda() && S.is_cuda() && R.is_contiguous() && S.is_contiguous(), "R, S on the device");
  TORCH_CHECK(mode >= 0 && mode <= 2, "mode is 0 (plain), 1 or 2 (pinned fractions)");
  TORCH_CHECK(frac > 0.0 && frac <= 1.0, "the pinned fraction must be in (0, 1]");
  TORCH_CHECK(grid > 0 && sink.numel() >= grid, "sink holds one word per CTA");
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(R.device());
    rc_ = sched_probe_mix(R.data_ptr(), R.numel() * R.element_size(), S.data_ptr(), S.numel() * S.element_size(),
                             mode, (float)frac, reinterpret_cast<unsigned *>(sink.data_ptr()), grid, cur_stream());
  }
  check_rc(rc_, "probe_mix");
}

void probe_pdl_pairs(at::Tensor &buf, at::Tensor &out, const at::Tensor &table, int64_t work, int64_t prologue,
                     bool pdl, int64_t pairs) {
  TORCH_CHECK(buf.is_cuda() && buf.scalar_type() == at::kFloat && out.sizes() == buf.sizes() &&
                  out.scalar_type() == at::kFloat && table.numel() >= 256 && table.scalar_type() == at::kFloat,
              "float32 buf/out of one shape and a float32 table of >= 256 entries");
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(buf.device());
    rc_ = sched_probe_pdl_pairs(buf.data_ptr<float>(), out.data_ptr<float>(), buf.numel(), table.data_ptr<float>(),
                                   work, prologue, pdl ? 1 : 0, pairs, cur_stream());
  }
  check_rc(rc_, "probe_pdl_pairs");
}

void probe_pdl_produce(at::Tensor &buf, int64_t work) {
  TORCH_CHECK(buf.is_cuda() && buf.scalar_type() == at::kFloat && buf.is_contiguous(), "float32 buf");
  int rc_ = 0;
  {  // the guard is gone before check_rc may throw
    c10::cuda::CUDAGuard g(buf.device());
    rc_ = sched_probe_pdl_produce(buf.data_ptr<float>(), buf.numel(), work, cur_stream());
  }
  check_rc(rc_, "probe_pdl_produce");
}

// Page moves between KV pools (device <-> pinned host); pairs [n, 2] int32 on the device.
// With n_dev (int32 [1] on the device) n_pairs is a capacity and the count is read there.
void kv_page_copy(const at::Tensor &src_k, const at::Tensor &src_v, at::Tensor &dst_k, at::Tensor &dst_v,
                  const at::Tensor &pairs, int64_t n_pairs, const c10::optional<at::Tensor> &n_dev,
                  const c10::optional<at::Tensor> &status) {
  TORCH_CHECK(src_k.dim() == 5 && dst_k.dim() == 5, "pools are [layers, pages, heads, 16, 128]");
  TORCH_CHECK(src_k.size(0) == dst_k.size(0) && src_k.size(2) == dst_k.size(2), "pool shapes differ");
  TORCH_CHECK(src_k.is_contiguous() && src_v.is_contiguous() && dst_k.is_contiguous() && dst_v.is_contiguous(),
              "contiguous pools");
  TORCH_CHECK(pairs.is_cuda() && pairs.scalar_type() == at::kInt && pairs.is_contiguous(), "pairs int32 on device");
  check_rc(sched_kv_page_copy(src_k.data_ptr(), src_v.data_ptr(), src_k.size(1), dst_k.data_ptr(), dst_v.data_ptr(),
                              dst_k.size(1), pairs.data_ptr<int32_t>(), n_pairs, ptr_or_null<int>(n_dev),
                              src_k.size(0), src_k.size(2), ptr_or_null<int>(status), cur_stream()),
           "kv_page_copy");
}

// Page moves between a bf16 pool and an fp8 (uint8 storage) pool; the scales
// [layers, fp8 pool pages, heads] fp32 belong to the fp8 pool.
void kv_page_copy_fp8(const at::Tensor &src_k, const at::Tensor &src_v, at::Tensor &dst_k, at::Tensor &dst_v,
                      at::Tensor &scale_k, at::Tensor &scale_v, bool to_fp8, const at::Tensor &pairs,
                      int64_t n_pairs, const c10::optional<at::Tensor> &n_dev,
                      const c10::optional<at::Tensor> &status) {
  TORCH_CHECK(src_k.dim() == 5 && dst_k.dim() == 5, "pools are [layers, pages, heads, 16, 128]");
  TORCH_CHECK(src_k.size(0) == dst_k.size(0) && src_k.size(2) == dst_k.size(2), "pool shapes differ");
  TORCH_CHECK(src_k.size(3) == 16 && src_k.size(4) == 128 && dst_k.size(3) == 16 && dst_k.size(4) == 128,
              "pages of 16 tokens x head dim 128");
  TORCH_CHECK(src_k.is_contiguous() && src_v.is_contiguous() && dst_k.is_contiguous() && dst_v.is_contiguous() &&
                  scale_k.is_contiguous() && scale_v.is_contiguous(),
              "contiguous pools");
  const at::Tensor &q = to_fp8 ? dst_k : src_k;
  const at::Tensor &b = to_fp8 ? src_k : dst_k;
  TORCH_CHECK(q.element_size() == 1 && b.scalar_type() == at::kBFloat16, "an fp8 (1-byte) pool and a bf16 pool");
  TORCH_CHECK(scale_k.scalar_type() == at::kFloat && scale_k.numel() == q.size(0) * q.size(1) * q.size(2) &&
                  scale_v.numel() == scale_k.numel(),
              "scales [layers, fp8 pages, heads] float32");
  TORCH_CHECK(pairs.is_cuda() && pairs.scalar_type() == at::kInt && pairs.is_contiguous(), "pairs int32 on device");
  check_rc(sched_kv_page_copy_fp8(src_k.data_ptr(), src_v.data_ptr(), src_k.size(1), dst_k.data_ptr(),
                                  dst_v.data_ptr(), dst_k.size(1), scale_k.data_ptr<float>(),
                                  scale_v.data_ptr<float>(), to_fp8 ? 1 : 0, pairs.data_ptr<int32_t>(), n_pairs,
                                  ptr_or_null<int>(n_dev), src_k.size(0), src_k.size(2), ptr_or_null<int>(status),
                                  cur_stream()),
           "kv_page_copy_fp8");
}

}  // namespace

void register_symm(py::module &m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  register_symm(m);
  m.def("take_error", &take_error);
  m.def("gemm_allreduce", &gemm_allreduce);
  m.def("gemm_reduce_scatter", &gemm_reduce_scatter);
  m.def("sp_reduce_norm", &sp_reduce_norm);
  m.def("sp_wait_rows", &sp_wait_rows);
  m.doc() = "sched_pass_b200 sm_100a kernels";
  m.def("gemm", &gemm);
  m.def("gemm_qkv_rope", &gemm_qkv_rope);
  m.def("gemm_ws_floats", &gemm_ws_floats);
  m.def("attn_decode", &attn_decode);
  m.def("attn_merge", &attn_merge);
  m.def("attn_prefill", &attn_prefill);
  m.def("attn_prefill_tile_rows", &sched_attn_prefill_tile_rows);
  m.def("attn_decode_occupancy", &attn_decode_occupancy);
  m.def("attn_decode_smem_bytes", &attn_decode_smem_bytes);
  m.def("add_rmsnorm", &add_rmsnorm);
  m.def("rope_kv_append", &rope_kv_append);
  m.def("embedding", &embedding);
  m.def("argmax", &argmax);
  m.def("argmax_exchange", &argmax_exchange);
  m.def("set_gemm_trace", &set_gemm_trace);
  m.def("set_attn_trace", &set_attn_trace);
  m.def("gemm_plan", [](int64_t T, int64_t N, int64_t K, int64_t epi, int64_t sms) {
    int cs = 0, grid = 0;
    sched_gemm_plan(T, N, K, epi, sms, &cs, &grid);
    return std::make_tuple(cs, grid);
  });
  m.def("gemm_pair_plan", [](int64_t T, int64_t N, int64_t K, int64_t epi, int64_t ws_floats, int64_t counters) {
    int np = 0, whole = 0, splits = 1;
    sched_gemm_pair_plan(T, N, K, epi, ws_floats, counters, &np, &whole, &splits);
    return std::make_tuple(np, whole, splits);
  });
  m.def("moe_router", &moe_router);
  m.def("kv_page_copy", &kv_page_copy);
  m.def("probe_stream", &probe_stream);
  m.def("probe_tasks", &probe_tasks);
  m.def("probe_tasks_occupancy", &sched_probe_tasks_occupancy);
  m.def("probe_mix", &probe_mix);
  m.def("probe_clc", &probe_clc);
  m.def("probe_clc_shape", &probe_clc_shape);
  m.def("probe_clc_shape_capacity", &sched_probe_clc_shape_capacity);
  m.def("kv_page_copy_fp8", &kv_page_copy_fp8);
  m.def("probe_pdl_pairs", &probe_pdl_pairs);
  m.def("probe_pdl_produce", &probe_pdl_produce);
  m.def("moe_dispatch", &moe_dispatch);
  m.def("moe_expert_gemm", &moe_expert_gemm);
  m.def("moe_quantize", &moe_quantize);
  m.def("moe_combine_norm", &moe_combine_norm);
}
