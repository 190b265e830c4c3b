// host_app_sched_rt.cu -- a host application on the named-global ABI
// (include/sched/sched_rt.h): it arms the control tables, programs a
// reversed task order and the timer, launches a kernel that reads the tables
// the way an IR-woven kernel does (pi with the order-size guard, timer rows),
// disarms, launches again (stock path), and prints the JSON publication.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -Iinclude -o host_app examples/host_app_sched_rt.cu
//   ./host_app                                   (needs a GPU)
#include <cstdio>
#include <vector>

#include "sched/sched_rt.h"

__global__ void demo(int *out, int n) {
  const int raw = blockIdx.x;
  int task = raw;
  const SchedCtrl *c = __sched_ctrl;
  if (__sched_task_order != nullptr && raw < SCHED_MAX_TASKS) {
    const int mapped = __sched_task_order[raw];
    const unsigned osz = c ? c->order_size : 0u;
    if (mapped >= 0 && mapped < n && (osz == 0u || osz == (unsigned)n)) task = mapped;
  }
  if (threadIdx.x == 0) {
    out[task] = 2 * task;
    const bool off = c ? (c->flags & SCHED_CTRL_FLAG_TIMER_OFF) != 0u : true;
    if (__sched_timer != nullptr && !off) atomicAdd(__sched_timer + task, 1ull);
  }
}

int main() {
  const int n = 64;
  if (!sched_rt_init()) return 1;
  std::vector<int32_t> rev(n);
  for (int i = 0; i < n; ++i) rev[i] = n - 1 - i;
  sched_rt_set_order(rev.data(), n);
  sched_rt_set_order_size(n);
  sched_rt_set_num_tasks(n);
  sched_rt_set_timer_enabled(true);
  if (!sched_rt_push_ctrl()) return 1;
  int *out = nullptr;
  cudaMalloc(&out, n * sizeof(int));
  std::vector<int> h(n);
  int bad = 0;
  for (int armed = 1; armed >= 0; --armed) {
    if (!armed) sched_rt_disarm();
    cudaMemset(out, 0xff, n * sizeof(int));
    demo<<<n, 32>>>(out, n);
    cudaDeviceSynchronize();
    cudaMemcpy(h.data(), out, n * sizeof(int), cudaMemcpyDeviceToHost);
    for (int i = 0; i < n; ++i) bad += h[i] != 2 * i;
  }
  // armed launch: one timer row per task; the disarmed launch wrote none
  for (int i = 0; i < n; ++i) bad += sched_rt_timer(i) != 1ull;
  char path[128];
  std::snprintf(path, sizeof(path), "/tmp/sched_rt_%d.json", (int)getpid());
  if (FILE *f = std::fopen(path, "r")) {
    char buf[512] = {0};
    std::fread(buf, 1, sizeof(buf) - 1, f);
    std::fclose(f);
    std::printf("%s", buf);
  } else {
    ++bad;
  }
  std::printf("%s\n", bad ? "FAIL" : "OK");
  return bad ? 1 : 0;
}
