// workqueue_pass.cpp -- the sched-workqueue pass: persistent-worker driver.
//
// Behaviour of the reference transform (lib/SchedWorkQueue.cpp:345-448):
// the kernel body is cloned into `<k>.sched_body(args..., i32 task)` with the
// task-axis ctaid replaced by the parameter, and the kernel becomes a driver:
//
//   armed (ctrl [+ queue]) and 1-D grid?        no -> stock: body(remap(ctaid))
//   num_tasks == 0 (per-step disarm)?          yes -> stock
//   ctaid >= num_tasks (surplus CTA)?          yes -> exit
//   loop: body(remap(raw)); barrier; thread 0 claims the next raw id
//         (ticket: atomic add on the queue; CLC: clusterlaunchcontrol
//         try_cancel of an unlaunched CTA); barrier; raw < num_tasks ? loop
//
// The claim comes after the body (late binding). The CLC claim's mbarrier
// wait is bounded: when the response never arrives within the spin limit the
// claim reports "no more work", so a lost response cannot hang the kernel.
#include <sstream>

#include "passes.h"

namespace weave {

namespace {

bool selected(const Config &c, const std::string &name) {
  if (c.wq_kernels.empty()) return true;
  std::stringstream ss(c.wq_kernels);
  std::string part;
  while (std::getline(ss, part, ','))
    if (!trim(part).empty() && name.find(trim(part)) != std::string::npos) return true;
  return false;
}

std::string join_args(const Function &f) {
  std::string s;
  for (size_t i = 0; i < f.param_names.size(); ++i) {
    if (i) s += ", ";
    s += f.param_types[i] + " " + f.param_names[i];
  }
  return s;
}

// remap inside the driver: clamp to num_tasks, honour order_size == num_tasks
std::string driver_remap(Function &f, std::vector<Inst> &e, Module &m, const Config &c, const Slot &order,
                         const std::string &ctrl, const std::string &raw, const std::string &ntasks) {
  if (!order.available || !c.pi) return raw;
  std::string zero = zero_table(m);
  std::string inb = f.unique("%sched.raw.inb"), use = f.unique("%sched.order.use");
  e.push_back(I("  " + inb + " = icmp ult i32 " + raw + ", " + std::to_string(c.max_tasks)));
  e.push_back(I("  " + use + " = and i1 " + order.armed + ", " + inb));
  std::string base = f.unique("%sched.order.base"), idx = f.unique("%sched.order.idx");
  std::string gep = f.unique("%sched.order.gep"), mapped = f.unique("%sched.task.mapped");
  e.push_back(I("  " + base + " = select i1 " + use + ", ptr " + order.ptr + ", ptr " + zero));
  e.push_back(I("  " + idx + " = select i1 " + use + ", i32 " + raw + ", i32 0"));
  e.push_back(I("  " + gep + " = getelementptr i32, ptr " + base + ", i32 " + idx));
  e.push_back(I("  " + mapped + " = load i32, ptr " + gep + ", align 4"));
  std::string osp = f.unique("%sched.order.size.p"), osz = f.unique("%sched.order.size");
  std::string u = f.unique("%sched.order.unchecked"), mt = f.unique("%sched.order.match");
  std::string valid = f.unique("%sched.order.valid"), ing = f.unique("%sched.task.ingrid");
  std::string ok = f.unique("%sched.task.ok"), ok2 = f.unique("%sched.task.ok"), task = f.unique("%sched.task");
  e.push_back(I("  " + osp + " = getelementptr i8, ptr " + ctrl + ", i64 28"));
  e.push_back(I("  " + osz + " = load i32, ptr " + osp + ", align 4"));
  e.push_back(I("  " + u + " = icmp eq i32 " + osz + ", 0"));
  e.push_back(I("  " + mt + " = icmp eq i32 " + osz + ", " + ntasks));
  e.push_back(I("  " + valid + " = or i1 " + u + ", " + mt));
  e.push_back(I("  " + ing + " = icmp ult i32 " + mapped + ", " + ntasks));
  e.push_back(I("  " + ok + " = and i1 " + ing + ", " + valid));
  e.push_back(I("  " + ok2 + " = and i1 " + ok + ", " + use));
  e.push_back(I("  " + task + " = select i1 " + ok2 + ", i32 " + mapped + ", i32 " + raw));
  return task;
}

bool transform(Module &m, Function &k, const Config &c, Notes &n) {
  const std::string slot_sreg = std::string("ctaid.") + "xyz"[c.slot_axis];
  // needs ctrl (and the queue for tickets): named global or baked address
  bool has_ctrl = m.has_global("@__sched_ctrl") || c.bake_ctrl;
  bool has_queue = m.has_global("@__sched_queue") || c.bake_queue;
  if (!has_ctrl || (!c.clc && !has_queue)) {
    n.add(k.name + ": work queue declined -- runtime slots not available");
    return false;
  }
  // ---- 1. clone the body: internal function with a trailing task argument
  Function body = k;
  body.name = k.name + ".sched_body";
  std::string task_arg = body.unique("%sched.task.arg");
  body.param_types.push_back("i32");
  body.param_names.push_back(task_arg);
  {
    std::string h = k.header;
    size_t at = h.find("@" + k.name + "(");
    size_t close = h.find(')', at);
    std::string params = h.substr(at + k.name.size() + 2, close - at - k.name.size() - 2);
    std::string attrs = trim(h.substr(close + 1));
    if (!attrs.empty() && attrs.back() == '{') attrs = trim(attrs.substr(0, attrs.size() - 1));
    body.header = "define internal void @" + body.name + "(" + params + (trim(params).empty() ? "" : ", ") +
                  "i32 " + task_arg + ") " + attrs + (attrs.empty() ? "" : " ") + kTaskBody + " {";
  }
  body.is_kernel = false;
  std::string slot_fn = "@llvm.nvvm.read.ptx.sreg." + slot_sreg + "()";
  for (Block &b : body.blocks) {
    std::vector<std::string> olds;
    for (auto it = b.insts.begin(); it != b.insts.end();) {
      if (it->opcode == "call" && it->text.find(slot_fn) != std::string::npos && !it->result.empty()) {
        olds.push_back(it->result);
        it = b.insts.erase(it);
      } else {
        ++it;
      }
    }
    for (const std::string &o : olds)
      for (Block &b2 : body.blocks)
        for (Inst &in : b2.insts) replace_uses(in, o, task_arg);
  }
  // ---- 2. rebuild the kernel as the driver
  Function d;
  d.name = k.name;
  d.is_kernel = true;
  d.param_types = k.param_types;
  d.param_names = k.param_names;
  for (const std::string &p : k.param_names) d.names.insert(p);
  {
    std::string h = k.header;
    size_t brace = h.rfind('{');
    d.header = h.substr(0, brace) + kWqDriver + " " + kInstrumented + " {";
  }
  std::string shared_next = "@" + k.name + ".sched_wq_next";
  m.add_global(shared_next + " = internal addrspace(3) global i32 undef, align 4");
  declare_sreg(m, slot_sreg);
  declare_sreg(m, "nctaid.y");
  declare_sreg(m, "nctaid.z");
  declare_sreg(m, "tid.x");
  declare_sreg(m, "tid.y");
  declare_sreg(m, "tid.z");
  m.add_declaration("declare void @llvm.nvvm.barrier0()");
  std::string args = join_args(k);

  Block entry, stock, dyn, bound, loop, claim, claimed, exitb;
  entry.label = "entry";
  stock.label = "sched.stock";
  dyn.label = "sched.dyn";
  bound.label = "sched.bound";
  loop.label = "sched.loop";
  claim.label = "sched.claim";
  claimed.label = "sched.claimed";
  exitb.label = "sched.exit";
  auto &e = entry.insts;
  Slot ctrl = load_slot(d, e, m, c, "@__sched_ctrl", c.bake_ctrl);
  Slot queue = c.clc ? Slot() : load_slot(d, e, m, c, "@__sched_queue", c.bake_queue);
  Slot order = load_slot(d, e, m, c, "@__sched_task_order", c.bake_order);
  std::string zero = zero_table(m);
  std::string ctrl_ptr = d.unique("%sched.ctrl");
  e.push_back(I("  " + ctrl_ptr + " = select i1 " + ctrl.armed + ", ptr " + ctrl.ptr + ", ptr " + zero));
  std::string first = d.unique("%sched.first");
  e.push_back(I("  " + first + " = call i32 @llvm.nvvm.read.ptx.sreg." + slot_sreg + "()"));
  const char *other1 = c.slot_axis == 0 ? "nctaid.y" : (c.slot_axis == 1 ? "nctaid.z" : "nctaid.x");
  const char *other2 = c.slot_axis == 0 ? "nctaid.z" : (c.slot_axis == 1 ? "nctaid.x" : "nctaid.y");
  declare_sreg(m, other1);
  declare_sreg(m, other2);
  std::string n1 = d.unique("%sched.n1"), n2 = d.unique("%sched.n2"), g1 = d.unique("%sched.g1"), g2 = d.unique("%sched.g2");
  std::string grid1d = d.unique("%sched.grid1d"), armed = d.unique("%sched.wq.armed");
  e.push_back(I("  " + n1 + " = call i32 @llvm.nvvm.read.ptx.sreg." + other1 + "()"));
  e.push_back(I("  " + n2 + " = call i32 @llvm.nvvm.read.ptx.sreg." + other2 + "()"));
  e.push_back(I("  " + g1 + " = icmp eq i32 " + n1 + ", 1"));
  e.push_back(I("  " + g2 + " = icmp eq i32 " + n2 + ", 1"));
  e.push_back(I("  " + grid1d + " = and i1 " + g1 + ", " + g2));
  std::string arm0 = c.clc ? ctrl.armed : d.unique("%sched.wq.slots");
  if (!c.clc) e.push_back(I("  " + arm0 + " = and i1 " + ctrl.armed + ", " + queue.armed));
  e.push_back(I("  " + armed + " = and i1 " + arm0 + ", " + grid1d));
  e.push_back(I("  br i1 " + armed + ", label %sched.dyn, label %sched.stock"));

  // stock: one task per CTA, pi still applies (identity when unarmed)
  {
    std::string nt = d.unique("%sched.ntiles");
    declare_sreg(m, "n" + slot_sreg);
    stock.insts.push_back(I("  " + nt + " = call i32 @llvm.nvvm.read.ptx.sreg.n" + slot_sreg + "()"));
    std::string t = driver_remap(d, stock.insts, m, c, order, ctrl_ptr, first, nt);
    stock.insts.push_back(I("  call void @" + body.name + "(" + args + (args.empty() ? "" : ", ") + "i32 " + t + ")"));
    stock.insts.push_back(I("  ret void"));
  }
  // dyn: num_tasks == 0 -> stock (per-step disarm, and the baked-ABI fail-safe)
  std::string ntp = d.unique("%sched.ntasks.p"), nts = d.unique("%sched.ntasks"), z = d.unique("%sched.ntasks.zero");
  dyn.insts.push_back(I("  " + ntp + " = getelementptr i8, ptr " + ctrl_ptr + ", i64 4"));
  dyn.insts.push_back(I("  " + nts + " = load i32, ptr " + ntp + ", align 4"));
  dyn.insts.push_back(I("  " + z + " = icmp eq i32 " + nts + ", 0"));
  dyn.insts.push_back(I("  br i1 " + z + ", label %sched.stock, label %sched.bound"));
  std::string sur = d.unique("%sched.surplus");
  bound.insts.push_back(I("  " + sur + " = icmp uge i32 " + first + ", " + nts));
  bound.insts.push_back(I("  br i1 " + sur + ", label %sched.exit, label %sched.loop"));
  // loop
  std::string raw = d.unique("%sched.raw"), next = d.unique("%sched.raw.next");
  loop.insts.push_back(I("  " + raw + " = phi i32 [ " + first + ", %sched.bound ], [ " + next + ", %sched.claimed ]"));
  std::string t = driver_remap(d, loop.insts, m, c, order, ctrl_ptr, raw, nts);
  loop.insts.push_back(I("  call void @" + body.name + "(" + args + (args.empty() ? "" : ", ") + "i32 " + t + ")"));
  loop.insts.push_back(I("  call void @llvm.nvvm.barrier0()"));
  std::string tx = d.unique("%sched.tid.x"), ty = d.unique("%sched.tid.y"), tz = d.unique("%sched.tid.z");
  std::string o1 = d.unique("%sched.tid.or"), o2 = d.unique("%sched.tid.or"), tzero = d.unique("%sched.tid.zero");
  loop.insts.push_back(I("  " + tx + " = call i32 @llvm.nvvm.read.ptx.sreg.tid.x()"));
  loop.insts.push_back(I("  " + ty + " = call i32 @llvm.nvvm.read.ptx.sreg.tid.y()"));
  loop.insts.push_back(I("  " + tz + " = call i32 @llvm.nvvm.read.ptx.sreg.tid.z()"));
  loop.insts.push_back(I("  " + o1 + " = or i32 " + tx + ", " + ty));
  loop.insts.push_back(I("  " + o2 + " = or i32 " + o1 + ", " + tz));
  loop.insts.push_back(I("  " + tzero + " = icmp eq i32 " + o2 + ", 0"));
  loop.insts.push_back(I("  br i1 " + tzero + ", label %sched.claim, label %sched.claimed"));
  // claim (thread 0), late binding
  std::string claimed_v = d.unique("%sched.claimed.raw");
  if (c.clc) {
    std::string res = "@" + k.name + ".sched_clc_res", bar = "@" + k.name + ".sched_clc_bar";
    m.add_global(res + " = internal addrspace(3) global [16 x i8] undef, align 16");
    m.add_global(bar + " = internal addrspace(3) global i64 undef, align 8");
    std::string ra = d.unique("%sched.clc.res"), ba = d.unique("%sched.clc.bar");
    claim.insts.push_back(I("  " + ra + " = ptrtoint ptr addrspace(3) " + res + " to i64"));
    claim.insts.push_back(I("  " + ba + " = ptrtoint ptr addrspace(3) " + bar + " to i64"));
    // try_cancel + bounded mbarrier wait + decode; the fallback (num_tasks
    // snapshot) ends the loop when no CTA is left or the wait gives up
    std::string asm_text =
        "{ .reg .pred %pc; .reg .pred %pl; .reg .b128 %rq; .reg .b64 %tmp; .reg .b32 %cx; .reg .b32 %cnt; "
        "mov.u32 %cx, $3; mov.u32 %cnt, 0; "
        "mbarrier.init.shared::cta.b64 [$2], 1; fence.proxy.async.shared::cta; "
        "mbarrier.arrive.expect_tx.shared::cta.b64 %tmp, [$2], 16; "
        "clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [$1], [$2]; "
        "sched_clc_wait${:uid}: mbarrier.try_wait.parity.shared::cta.b64 %pc, [$2], 0; "
        "@%pc bra sched_clc_done${:uid}; add.u32 %cnt, %cnt, 1; setp.lt.u32 %pl, %cnt, " +
        std::to_string(c.clc_spin_limit) +
        "; @%pl bra sched_clc_wait${:uid}; bra sched_clc_out${:uid}; "
        "sched_clc_done${:uid}: ld.shared.b128 %rq, [$1]; "
        "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 %pc, %rq; "
        "@%pc clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %cx, %rq; "
        "sched_clc_out${:uid}: mov.u32 $0, %cx; }";
    claim.insts.push_back(I("  " + claimed_v + " = call i32 asm sideeffect \"" + asm_text +
                            "\", \"=r,l,l,r,~{memory}\"(i64 " + ra + ", i64 " + ba + ", i32 " + nts + ")"));
  } else {
    claim.insts.push_back(I("  " + claimed_v + " = atomicrmw add ptr " + queue.ptr + ", i32 1 monotonic, align 4"));
  }
  claim.insts.push_back(I("  store i32 " + claimed_v + ", ptr addrspace(3) " + shared_next + ", align 4"));
  claim.insts.push_back(I("  br label %sched.claimed"));
  claimed.insts.push_back(I("  call void @llvm.nvvm.barrier0()"));
  claimed.insts.push_back(I("  " + next + " = load i32, ptr addrspace(3) " + shared_next + ", align 4"));
  std::string done = d.unique("%sched.done");
  claimed.insts.push_back(I("  " + done + " = icmp uge i32 " + next + ", " + nts));
  claimed.insts.push_back(I("  br i1 " + done + ", label %sched.exit, label %sched.loop"));
  exitb.insts.push_back(I("  ret void"));
  d.blocks = {entry, stock, dyn, bound, loop, claim, claimed, exitb};

  // place the body clone right after the driver
  for (size_t i = 0; i < m.functions.size(); ++i)
    if (m.functions[i].name == k.name) {
      m.functions[i] = d;
      m.functions.push_back(body);
      for (size_t li = 0; li < m.lines.size(); ++li)
        if (m.lines[li] == kFuncMark + std::to_string(i)) {
          m.lines.insert(m.lines.begin() + li + 1, kFuncMark + std::to_string(m.functions.size() - 1));
          break;
        }
      break;
    }
  n.add(k.name + ": work-queue driver built (" + std::string(c.clc ? "cluster launch control" : "ticket") +
        " claim, late-bound)");
  return true;
}

}  // namespace

bool run_workqueue(Module &m, const Config &c, Notes &notes) {
  if (!c.workqueue) return false;
  std::vector<std::string> names;
  for (const Function &f : m.functions)
    if (f.is_kernel && selected(c, f.name) && f.header.find(kWqDriver) == std::string::npos) names.push_back(f.name);
  bool changed = false;
  for (const std::string &nm : names)
    for (Function &f : m.functions)
      if (f.name == nm) {
        Function copy = f;
        changed |= transform(m, copy, c, notes);
        break;
      }
  return changed;
}

}  // namespace weave
