// gemm_c_api.cpp -- calling the tcgen05 GEMM from C++ through the torch-free
// kernel library (libsched_kernels, built by CMake with
// -DSCHED_BUILD_KERNELS=ON). Computes y = x . w^T for a decode-sized shape,
// checks it against a float reference on the host, and prints the error.
//
//   cmake -S . -B build -DSCHED_BUILD_KERNELS=ON && cmake --build build
//   ./build/sched_example_gemm            (needs a B200)
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <random>
#include <vector>

#include "gemm_api.h"

#define CHECK(x)                                                                 \
  do {                                                                           \
    cudaError_t e_ = (x);                                                        \
    if (e_ != cudaSuccess) {                                                     \
      std::fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));              \
      return 1;                                                                  \
    }                                                                            \
  } while (0)

int main() {
  const int T = 16, N = 1024, K = 2048;
  std::mt19937 rng(0);
  std::normal_distribution<float> nd(0.f, 1.f);
  std::vector<__nv_bfloat16> hx(T * K), hw(N * K);
  for (auto &v : hx) v = __float2bfloat16(nd(rng));
  for (auto &v : hw) v = __float2bfloat16(nd(rng) / std::sqrt((float)K));

  __nv_bfloat16 *x, *w, *y;
  int *status;
  CHECK(cudaMalloc(&x, hx.size() * 2));
  CHECK(cudaMalloc(&w, hw.size() * 2));
  CHECK(cudaMalloc(&y, (size_t)T * N * 2));
  CHECK(cudaMalloc(&status, 16));
  CHECK(cudaMemset(status, 0, 16));
  CHECK(cudaMemcpy(x, hx.data(), hx.size() * 2, cudaMemcpyHostToDevice));
  CHECK(cudaMemcpy(w, hw.data(), hw.size() * 2, cudaMemcpyHostToDevice));

  // stream-K scratch: partial slices (sized by the library) and tile counters (zeroed once)
  const long long ws_floats = sched_gemm_ws_floats(T, N, K, 0);
  float *ws = nullptr;
  uint32_t *counters = nullptr;
  const int n_counters = 1 << 12;
  if (ws_floats > 0) CHECK(cudaMalloc(&ws, ws_floats * 4));
  CHECK(cudaMalloc(&counters, n_counters * 4));
  CHECK(cudaMemset(counters, 0, n_counters * 4));

  GemmArgs a{};
  a.x = x;
  a.ldx = K;
  a.w = w;
  a.y = y;
  a.ldy = N;
  a.T = T;
  a.N = N;
  a.K = K;
  a.epi = kEpiStore;
  a.num_sms = 148;
  a.ws = ws;
  a.ws_floats = ws_floats;
  a.counters = counters;
  a.counter_count = n_counters;
  a.status = status;
  const int rc = sched_gemm_run(&a, 0);
  if (rc != 0) {
    std::fprintf(stderr, "sched_gemm_run: code %d\n", rc);
    return 1;
  }
  CHECK(cudaDeviceSynchronize());
  int st[4];
  CHECK(cudaMemcpy(st, status, 16, cudaMemcpyDeviceToHost));
  std::vector<__nv_bfloat16> hy((size_t)T * N);
  CHECK(cudaMemcpy(hy.data(), y, hy.size() * 2, cudaMemcpyDeviceToHost));

  double err = 0, ref_norm = 0;
  for (int t = 0; t < T; ++t)
    for (int n = 0; n < N; ++n) {
      float r = 0.f;
      for (int k = 0; k < K; ++k) r += __bfloat162float(hx[t * K + k]) * __bfloat162float(hw[n * K + k]);
      const double d = __bfloat162float(hy[(size_t)t * N + n]) - r;
      err += d * d;
      ref_norm += (double)r * r;
    }
  std::printf("status %d, relative error %.3e\n", st[0], std::sqrt(err / ref_norm));
  return (st[0] == 0 && std::sqrt(err / ref_norm) < 1e-2) ? 0 : 1;
}
