// passes.cpp -- weave configuration and the emission helpers both passes use.
#include <cstdlib>
#include <cstring>
#include <sstream>

#include "passes.h"

namespace weave {

namespace {

int env_int(const char *k, int d) {
  const char *v = std::getenv(k);
  return v ? std::atoi(v) : d;
}
double env_f(const char *k, double d) {
  const char *v = std::getenv(k);
  return v ? std::atof(v) : d;
}
uint64_t env_addr(const char *k) {
  const char *v = std::getenv(k);
  return v ? std::strtoull(v, nullptr, 0) : 0ull;
}
bool env_on(const char *k) { return std::getenv(k) != nullptr; }

}  // namespace

Config Config::from_env() {
  Config c;
  c.slot_axis = env_int("SCHED_SLOT_AXIS", 0);
  if (c.slot_axis < 0 || c.slot_axis > 2) c.slot_axis = 0;
  int mt = env_int("SCHED_MAX_TASKS", 4096);
  c.max_tasks = (mt > 0 && mt <= (1 << 20)) ? (unsigned)mt : 4096u;
  c.pi = !env_on("SCHED_NO_INDIRECT");
  c.timer = !env_on("SCHED_NO_TIMER");
  c.policy = !env_on("SCHED_NO_POLICY");
  c.shed = !env_on("SCHED_NO_SHED");
  c.pdl = env_on("SCHED_PDL");
  c.workqueue = env_on("SCHED_WORKQUEUE");
  c.clc = env_on("SCHED_CLC");
  c.timer_indirect = env_on("SCHED_TIMER_INDIRECT");
  c.order_indirect = env_on("SCHED_ORDER_INDIRECT");
  c.prefetch_dist = (unsigned)env_int("SCHED_PF_DIST", 8);
  c.dT = env_f("SCHED_DT", 1.0);
  c.dR = env_f("SCHED_DR", 1.0);
  c.H = env_f("SCHED_H", 0.25);
  c.debug = env_on("SCHED_DEBUG");
  if (const char *w = std::getenv("SCHED_WQ_KERNELS")) c.wq_kernels = w;
  c.bake_order = env_addr("SCHED_BAKE_TASK_ORDER");
  c.bake_ctrl = env_addr("SCHED_BAKE_CTRL");
  c.bake_timer = env_addr("SCHED_BAKE_TIMER");
  c.bake_queue = env_addr("SCHED_BAKE_QUEUE");
  return c;
}

Inst I(const std::string &text) { return parse_inst(text); }

// Address space of a module-level global from its definition line.
static int global_addrspace(const Module &m, const std::string &g) {
  for (const std::string &l : m.lines)
    if (starts_with(l, g + " ") || starts_with(l, g + "=")) {
      size_t p = l.find("addrspace(");
      size_t eq = l.find('=');
      if (p != std::string::npos && (eq == std::string::npos || p < l.find("global", eq)))
        return std::atoi(l.c_str() + p + 10);
      return 0;
    }
  return 0;
}

Slot load_slot(Function &f, std::vector<Inst> &out, Module &m, const Config &c, const std::string &global,
               uint64_t baked) {
  Slot s;
  std::string base = global.substr(3);  // "__sched_ctrl" -> "sched_ctrl"
  if (m.has_global(global)) {
    int as = global_addrspace(m, global);
    std::string gp = as ? "ptr addrspace(" + std::to_string(as) + ") " + global : "ptr " + global;
    s.ptr = f.unique("%" + std::string("sched.") + base.substr(6) + ".slot");
    out.push_back(I("  " + s.ptr + " = load ptr, " + gp + ", align 8"));
    s.armed = f.unique("%" + std::string("sched.") + base.substr(6) + ".armed");
    out.push_back(I("  " + s.armed + " = icmp ne ptr " + s.ptr + ", null"));
    s.available = true;
  } else if (baked != 0) {
    // The address lives in a non-constant internal global so the compiler
    // cannot fold it into an immediate of every access.
    std::string bg = global + ".bakedslot";
    if (!m.has_global(bg))
      m.add_global(bg + " = internal addrspace(1) global i64 " + std::to_string(baked) + ", align 8");
    std::string v = f.unique("%sched." + base.substr(6) + ".baked");
    s.ptr = f.unique("%sched." + base.substr(6) + ".slot");
    out.push_back(I("  " + v + " = load i64, ptr addrspace(1) " + bg + ", align 8"));
    out.push_back(I("  " + s.ptr + " = inttoptr i64 " + v + " to ptr"));
    s.armed = "true";
    s.available = true;
  }
  (void)c;
  return s;
}

std::string zero_table(Module &m) {
  if (!m.has_global("@__sched.zero"))
    m.add_global("@__sched.zero = internal addrspace(1) global [64 x i64] zeroinitializer, align 16");
  return "addrspacecast (ptr addrspace(1) @__sched.zero to ptr)";
}

void declare_sreg(Module &m, const std::string &which) {
  std::string ty = which == "clock64" ? "i64" : "i32";
  m.add_declaration("declare " + ty + " @llvm.nvvm.read.ptx.sreg." + which + "()");
}

std::string sreg(Function &f, std::vector<Inst> &out, const std::string &which) {
  std::string v = f.unique("%sched.sreg." + which);
  std::string ty = which == "clock64" ? "i64" : "i32";
  out.push_back(I("  " + v + " = call " + ty + " @llvm.nvvm.read.ptx.sreg." + which + "()"));
  return v;
}

}  // namespace weave
