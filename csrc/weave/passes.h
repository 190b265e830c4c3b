// passes.h -- configuration and entry points of the two weaving passes.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "ir.h"

namespace weave {

// Weave-time configuration, read from the environment with the knob names of
// the manifest (sched/manifest.h) and the reference's bake protocol.
struct Config {
  int slot_axis = 0;            // SCHED_SLOT_AXIS: 0 x, 1 y, 2 z (the task axis)
  unsigned max_tasks = 4096;    // SCHED_MAX_TASKS (1 .. 2^20)
  bool pi = true;               // !SCHED_NO_INDIRECT
  bool timer = true;            // !SCHED_NO_TIMER
  bool policy = true;           // !SCHED_NO_POLICY
  bool shed = true;             // !SCHED_NO_SHED
  bool pdl = false;             // SCHED_PDL
  bool workqueue = false;       // SCHED_WORKQUEUE
  bool clc = false;             // SCHED_CLC (claim via cluster launch control)
  bool timer_indirect = false;  // SCHED_TIMER_INDIRECT: the timer slot holds a row-table pointer
  bool order_indirect = false;  // SCHED_ORDER_INDIRECT: the order slot holds a table pointer
  unsigned prefetch_dist = 8;   // SCHED_PF_DIST (iterations ahead)
  double dT = 1.0, dR = 1.0, H = 0.25;  // SCHED_DT / SCHED_DR / SCHED_H
  bool debug = false;           // SCHED_DEBUG
  std::string wq_kernels;       // SCHED_WQ_KERNELS: comma list of name substrings
  uint64_t bake_order = 0, bake_ctrl = 0, bake_timer = 0, bake_queue = 0;  // SCHED_BAKE_*
  unsigned clc_spin_limit = 1u << 22;  // bounded wait of the CLC claim

  static Config from_env();
};

struct Notes {
  std::vector<std::string> lines;
  bool debug = false;
  void add(const std::string &s) { lines.push_back(s); }
};

// Returns true when the module changed.
bool run_weave(Module &m, const Config &c, Notes &notes);
bool run_workqueue(Module &m, const Config &c, Notes &notes);

// Attribute markers (string function attributes).
constexpr const char *kInstrumented = "\"sched-instrumented\"";
constexpr const char *kTaskBody = "\"sched-task-body\"";
constexpr const char *kWqDriver = "\"sched-wq-driver\"";

// Shared emission helpers (passes.cpp).
struct Slot {
  bool available = false;
  std::string ptr;    // value holding the table pointer (generic "ptr")
  std::string armed;  // i1 value (or "true")
};
Slot load_slot(Function &f, std::vector<Inst> &out, Module &m, const Config &c,
               const std::string &global, uint64_t baked);
std::string zero_table(Module &m);
std::string sreg(Function &f, std::vector<Inst> &out, const std::string &which);
void declare_sreg(Module &m, const std::string &which);
Inst I(const std::string &text);

}  // namespace weave
