// weave_pass.cpp -- the sched-weave pass: pi, shed, policy, timer, PDL.
//
// Semantics (per manifest row, include/sched/manifest.h) follow the
// reference pass lib/SchedWeave.cpp (remap :444-526, policy flags :532-581,
// budget :585-614, shed :652-842, prefetch :863-922, PDL :947-960, timer
// :979-1049), re-implemented over the textual IR model:
//
//  * entry code is branch-free: a null slot selects a zero-filled internal
//    table instead of being branched around, so every table read is safe
//    and a disarmed kernel reads the neutral values (identity order, tau 0,
//    hint 0 / q 0, flags 0) -- the "null slots => stock" contract holds by
//    construction;
//  * the only control flow the pass adds is the timer's guarded atomic in
//    front of each `ret` (a block that has no successors, so no phi needs
//    updating);
//  * shed masks on the loop's canonical induction variable and declines
//    (with a note) on any loop or site it cannot prove the shape of.
#include <cctype>
#include <cstdlib>
#include <functional>
#include <map>
#include <sstream>

#include "cfg.h"
#include "passes.h"

namespace weave {

namespace {

std::string fmt_double(double v) {
  // LLVM float literals: use the exact double hex form
  union {
    double d;
    uint64_t u;
  } x;
  x.d = v;
  char buf[32];
  std::snprintf(buf, sizeof(buf), "0x%016llX", (unsigned long long)x.u);
  return buf;
}

const char *kNegInf = "0xFFF0000000000000";

int int_bits(const std::string &ty) {
  if (ty.size() > 1 && ty[0] == 'i') return std::atoi(ty.c_str() + 1);
  return 0;
}

bool is_float_ty(const std::string &t) { return t == "float" || t == "double" || t == "half" || t == "bfloat"; }

// Definition map of a function: value name -> (block index, inst index).
struct Defs {
  std::map<std::string, std::pair<int, int>> at;
  explicit Defs(const Function &f) {
    for (size_t b = 0; b < f.blocks.size(); ++b)
      for (size_t i = 0; i < f.blocks[b].insts.size(); ++i)
        if (!f.blocks[b].insts[i].result.empty()) at[f.blocks[b].insts[i].result] = {(int)b, (int)i};
  }
  const Inst *get(const Function &f, const std::string &v) const {
    auto it = at.find(v);
    if (it == at.end()) return nullptr;
    return &f.blocks[it->second.first].insts[it->second.second];
  }
};

std::string callee_of(const Inst &in) {
  if (in.opcode != "call") return "";
  size_t at = in.text.find('@');
  if (at == std::string::npos) return "";
  size_t e = at + 1;
  while (e < in.text.size() && (std::isalnum((unsigned char)in.text[e]) || in.text[e] == '.' || in.text[e] == '_'))
    ++e;
  return in.text.substr(at + 1, e - at - 1);
}

bool is_exp_call(const Inst &in) {
  std::string c = callee_of(in);
  if (c.empty()) return false;
  if (c.find("frexp") != std::string::npos || c.find("ldexp") != std::string::npos) return false;
  return c.find("exp") != std::string::npos || c.find("ex2") != std::string::npos;
}
bool is_max_call(const Inst &in) {
  std::string c = callee_of(in);
  return c.find("maxnum") != std::string::npos || (c.find("fmax") != std::string::npos && c.find("fmaxnan") == std::string::npos);
}
bool is_arith(const Inst &in) {
  static const std::set<std::string> k = {"fadd", "fsub", "fmul", "fdiv", "fneg", "select", "fpext", "fptrunc",
                                          "bitcast", "sitofp", "uitofp", "add", "sub", "mul"};
  if (k.count(in.opcode)) return true;
  if (in.opcode == "call") {  // fused multiply-add intrinsics carry the dot product
    std::string c = callee_of(in);
    return c.rfind("llvm.fma.", 0) == 0 || c.rfind("llvm.fmuladd.", 0) == 0;
  }
  return false;
}

// Users of a value (block, inst) in the function.
std::vector<std::pair<int, int>> users(const Function &f, const std::string &v) {
  std::vector<std::pair<int, int>> u;
  for (size_t b = 0; b < f.blocks.size(); ++b)
    for (size_t i = 0; i < f.blocks[b].insts.size(); ++i)
      if (uses(f.blocks[b].insts[i], v)) u.push_back({(int)b, (int)i});
  return u;
}

bool reaches_exp(const Function &f, const std::string &v) {
  std::vector<std::string> work{v};
  std::set<std::string> seen;
  int steps = 0;
  while (!work.empty() && steps++ < 64) {
    std::string cur = work.back();
    work.pop_back();
    if (!seen.insert(cur).second) continue;
    for (auto [b, i] : users(f, cur)) {
      const Inst &u = f.blocks[b].insts[i];
      if (is_exp_call(u)) return true;
      if (is_arith(u) && !u.result.empty()) work.push_back(u.result);
    }
  }
  return false;
}

// The online-softmax score derived from load `ld`: a value reached through
// arithmetic (and warp shuffles) that feeds a running max AND an exp.
std::string find_softmax_score(const Function &f, const std::string &ld) {
  std::vector<std::string> work{ld};
  std::set<std::string> seen;
  int steps = 0;
  while (!work.empty() && steps++ < 256) {
    std::string cur = work.back();
    work.pop_back();
    if (!seen.insert(cur).second) continue;
    for (auto [b, i] : users(f, cur)) {
      const Inst &u = f.blocks[b].insts[i];
      bool feeds_max = is_max_call(u) || u.opcode == "fcmp";
      if (feeds_max && cur != ld && reaches_exp(f, cur)) return cur;
      if (is_arith(u)) {
        if (!u.result.empty()) work.push_back(u.result);
        continue;
      }
      if (u.opcode == "call") {
        std::string c = callee_of(u);
        if (c.rfind("llvm.nvvm.shfl", 0) == 0 && !u.result.empty()) work.push_back(u.result);
        continue;
      }
      if ((is_arith(u) || u.opcode == "fpext") && !u.result.empty()) work.push_back(u.result);
    }
  }
  return "";
}

// Loops come from the CFG analysis (cfg.h): natural loops over the
// dominator tree, each with its structurally recognised canonical IV.
using Loop = NaturalLoop;

std::vector<Loop> find_loops(const Function &f) { return natural_loops(f, Cfg(f)); }

bool in_loop(const Loop &L, int b) { return L.contains(b); }

// Does `v` depend (within a few steps of address arithmetic) on a load
// inside the loop, or on the IV?
enum class Mu { None, Index, Arith };
Mu address_kind(const Function &f, const Defs &defs, const Loop &L, const std::string &ptr) {
  std::vector<std::string> work{ptr};
  std::set<std::string> seen;
  bool iv = false;
  int steps = 0;
  while (!work.empty() && steps++ < 64) {
    std::string cur = work.back();
    work.pop_back();
    if (!seen.insert(cur).second) continue;
    if (cur == L.iv) iv = true;
    const Inst *d = defs.get(f, cur);
    if (!d) continue;
    auto pos = defs.at.find(cur)->second;
    if (d->opcode == "load" && in_loop(L, pos.first)) return Mu::Index;
    if (d->opcode == "getelementptr" || d->opcode == "add" || d->opcode == "mul" || d->opcode == "shl" ||
        d->opcode == "sext" || d->opcode == "zext" || d->opcode == "trunc" || d->opcode == "or" ||
        d->opcode == "addrspacecast" || d->opcode == "sub")
      for (const std::string &o : d->operands) work.push_back(o);
  }
  return iv ? Mu::Arith : Mu::None;
}

// d(index)/d(iv) of an integer expression: only add/sub/mul/shl by constants
// and casts are understood; returns false otherwise.
bool iv_step(const Function &f, const Defs &defs, const std::string &iv, const std::string &v, long long &step,
             int depth = 0) {
  if (v == iv) {
    step = 1;
    return true;
  }
  if (depth > 12) return false;
  const Inst *d = defs.get(f, v);
  if (!d) {
    step = 0;
    return true;  // argument / constant
  }
  auto pos = defs.at.find(v)->second;
  (void)pos;
  const std::string &op = d->opcode;
  if (op == "sext" || op == "zext" || op == "trunc") return iv_step(f, defs, iv, d->operands.empty() ? "" : d->operands[0], step, depth + 1);
  if (op == "add" || op == "sub" || op == "mul" || op == "shl") {
    std::string t = d->text;
    size_t ty = t.find(d->type);
    std::string ops = t.substr(ty + d->type.size());
    size_t c = ops.find(',');
    std::string a = trim(ops.substr(0, c)), b = trim(ops.substr(c + 1));
    b = b.substr(0, b.find_first_of(" ,;"));
    auto val = [&](const std::string &x, long long &s, bool &is_const, long long &cv) -> bool {
      if (!x.empty() && x[0] == '%') {
        is_const = false;
        return iv_step(f, defs, iv, x, s, depth + 1);
      }
      is_const = true;
      cv = std::atoll(x.c_str());
      s = 0;
      return true;
    };
    long long sa, sb, ca = 0, cb = 0;
    bool ka, kb;
    if (!val(a, sa, ka, ca) || !val(b, sb, kb, cb)) return false;
    if (op == "add") step = sa + sb;
    else if (op == "sub") step = sa - sb;
    else if (op == "mul") {
      if (ka) step = ca * sb;
      else if (kb) step = cb * sa;
      else return sa == 0 && sb == 0 ? (step = 0, true) : false;
    } else {  // shl
      if (!kb) return false;
      step = sa << cb;
    }
    return true;
  }
  // any other definition inside the function: treat as loop-invariant only if
  // it does not transitively use the IV
  std::vector<std::string> work{v};
  std::set<std::string> seen;
  while (!work.empty()) {
    std::string cur = work.back();
    work.pop_back();
    if (!seen.insert(cur).second) continue;
    if (cur == iv) return false;
    const Inst *dd = defs.get(f, cur);
    if (dd && dd->opcode != "phi")
      for (const std::string &o : dd->operands) work.push_back(o);
  }
  step = 0;
  return true;
}

int type_bytes(const std::string &t) {
  if (t == "float" || t == "i32") return 4;
  if (t == "double" || t == "i64" || starts_with(t, "ptr")) return 8;
  if (t == "half" || t == "bfloat" || t == "i16") return 2;
  if (t == "i8") return 1;
  return 0;
}

// The base object a pointer is derived from (argument, global, or the first
// value the walk cannot see through).
std::string pointer_root(const Function &f, const Defs &defs, std::string v) {
  for (int steps = 0; steps < 32; ++steps) {
    const Inst *d = defs.get(f, v);
    if (!d || d->operands.empty()) return v;
    if (d->opcode == "getelementptr" || d->opcode == "addrspacecast" || d->opcode == "bitcast") {
      v = d->operands[0];
      continue;
    }
    return v;
  }
  return v;
}

// Roots of every pointer the function stores or atomically updates through:
// loads from these are not read-only streams (an L2 discard would drop dirty
// data, a value mask would corrupt an accumulator).
std::set<std::string> written_roots(const Function &f, const Defs &defs) {
  std::set<std::string> roots;
  for (const Block &b : f.blocks)
    for (const Inst &in : b.insts) {
      if (in.opcode == "store" && in.operands.size() >= 2) roots.insert(pointer_root(f, defs, in.operands.back()));
      if ((in.opcode == "atomicrmw" || in.opcode == "cmpxchg") && !in.operands.empty())
        roots.insert(pointer_root(f, defs, in.operands[0]));
    }
  return roots;
}

struct Site {
  int block, inst;
  std::string load, ptr, ptr_type, ty;
  Mu mu;
  int loop;
};

// A cp.async in a loop: its global source address is a stream the urgent
// tier can warm in L2 ahead of the copy (the reference's async stream sites,
// lib/SchedWeave.cpp:264-300 / :928-942). The data lands in shared memory,
// so it is neither value-masked nor demoted.
struct AsyncSite {
  std::string text;  // the call's line (its position is found again by text)
  std::string src, src_type;
  int loop;
};

// A TMA tensor load (cp.async.bulk.tensor, tile mode, global -> shared) in a
// loop: the stream the reference lists as not visible to its IR detectors
// (MODEL.md:100, "TMA descriptor ... not visible as plain loads at LLVM IR";
// lib/SchedWeave.cpp:155-160 leaves it to other observation levels). Here
// the load's inline asm names the descriptor and the box coordinates, so the
// site is visible. When a box coordinate advances with the canonical IV, the urgent tier
// prefetches the box `dist` iterations ahead into L2 with
// cp.async.bulk.prefetch.tensor on the advanced coordinates.
struct TmaSite {
  std::string text;
  int dims = 0;
  std::string tmap, tmap_type;      // the tensor-map operand
  std::vector<std::string> coords;  // i32 box coordinates, innermost first
  int loop = -1;
};

// Split "a, b(c, d), e" at top-level commas.
std::vector<std::string> split_top(const std::string &s) {
  std::vector<std::string> out;
  int depth = 0;
  std::string cur;
  for (char ch : s) {
    if (ch == '(' || ch == '{' || ch == '[' || ch == '<') ++depth;
    if (ch == ')' || ch == '}' || ch == ']' || ch == '>') --depth;
    if (ch == ',' && depth == 0) {
      out.push_back(trim(cur));
      cur.clear();
    } else {
      cur += ch;
    }
  }
  if (!trim(cur).empty()) out.push_back(trim(cur));
  return out;
}

// `call void asm sideeffect "<asm>", "<constraints>"(<args>)` holding a
// cp.async: the argument bound to a 64-bit ("l") constraint with pointer type
// is the global source. False when the line is not such a call.
bool parse_cp_async(const std::string &text, std::string &src, std::string &src_type) {
  const size_t a = text.find("asm ");
  if (a == std::string::npos || text.find("cp.async") == std::string::npos) return false;
  const size_t q0 = text.find('"', a);
  const size_t q1 = q0 == std::string::npos ? q0 : text.find('"', q0 + 1);
  const size_t c0 = q1 == std::string::npos ? q1 : text.find('"', q1 + 1);
  const size_t c1 = c0 == std::string::npos ? c0 : text.find('"', c0 + 1);
  if (c1 == std::string::npos) return false;
  const std::string asm_text = text.substr(q0 + 1, q1 - q0 - 1);
  if (asm_text.find("cp.async") == std::string::npos || asm_text.find("bulk") != std::string::npos) return false;
  std::vector<std::string> cons;
  for (const std::string &k : split_top(text.substr(c0 + 1, c1 - c0 - 1)))
    if (!starts_with(k, "~{") && !starts_with(k, "=")) cons.push_back(k);
  const size_t p0 = text.find('(', c1), p1 = text.rfind(')');
  if (p0 == std::string::npos || p1 == std::string::npos || p1 <= p0) return false;
  std::vector<std::string> args = split_top(text.substr(p0 + 1, p1 - p0 - 1));
  for (size_t i = 0; i < args.size() && i < cons.size(); ++i) {
    const size_t sp = args[i].rfind(' ');
    if (sp == std::string::npos) continue;
    const std::string ty = trim(args[i].substr(0, sp)), v = trim(args[i].substr(sp + 1));
    if (cons[i] == "l" && starts_with(ty, "ptr") && !v.empty() && v[0] == '%') {
      src = v;
      src_type = ty;
      return true;
    }
  }
  return false;
}

// `call void asm sideeffect "<asm>", "<constraints>"(<args>)` whose asm holds
// a tiled TMA load "cp.async.bulk.tensor.<N>d.shared...global... [dst],
// [$m, {$c0, ...}], ...": the tensor map is argument m (a 64-bit "l"
// operand), the coordinates the i32 arguments named inside the braces.
// False for any other line, for stores and reductions (global before
// shared), for im2col boxes and for prefetches.
bool parse_tma_load(const std::string &text, TmaSite &s) {
  const size_t a = text.find("asm ");
  if (a == std::string::npos || text.find("cp.async.bulk.tensor.") == std::string::npos) return false;
  const size_t q0 = text.find('"', a);
  const size_t q1 = q0 == std::string::npos ? q0 : text.find('"', q0 + 1);
  const size_t c0 = q1 == std::string::npos ? q1 : text.find('"', q1 + 1);
  const size_t c1 = c0 == std::string::npos ? c0 : text.find('"', c0 + 1);
  if (c1 == std::string::npos) return false;
  const std::string asm_text = text.substr(q0 + 1, q1 - q0 - 1);
  const size_t op = asm_text.find("cp.async.bulk.tensor.");
  if (op == std::string::npos) return false;
  const size_t op_end = asm_text.find_first_of(" \t[", op);
  if (op_end == std::string::npos) return false;
  const std::string opcode = asm_text.substr(op, op_end - op);
  const size_t dpos = std::string("cp.async.bulk.tensor.").size();
  if (opcode.size() < dpos + 2 || opcode[dpos + 1] != 'd') return false;
  const int dims = opcode[dpos] - '0';
  if (dims < 1 || dims > 5) return false;
  const size_t sh = opcode.find(".shared"), gl = opcode.find(".global");
  if (sh == std::string::npos || gl == std::string::npos || gl < sh) return false;  // loads only
  if (opcode.find("im2col") != std::string::npos || opcode.find("prefetch") != std::string::npos) return false;
  // the second bracketed operand: [$m, {$c0, ...}]
  const size_t b1 = asm_text.find('[', op_end), e1 = b1 == std::string::npos ? b1 : asm_text.find(']', b1);
  const size_t b2 = e1 == std::string::npos ? e1 : asm_text.find('[', e1);
  const size_t e2 = b2 == std::string::npos ? b2 : asm_text.find(']', b2);
  if (e2 == std::string::npos) return false;
  const std::string inner = asm_text.substr(b2 + 1, e2 - b2 - 1);
  const size_t lb = inner.find('{'), rb = inner.find('}');
  if (lb == std::string::npos || rb == std::string::npos || rb < lb) return false;
  auto operand_index = [](const std::string &tok) -> int {
    const std::string t = trim(tok);
    if (t.size() < 2 || t[0] != '$') return -1;
    for (size_t i = 1; i < t.size(); ++i)
      if (t[i] < '0' || t[i] > '9') return -1;
    return std::atoi(t.c_str() + 1);
  };
  const int mi = operand_index(inner.substr(0, inner.find(',')));
  std::vector<int> ci;
  for (const std::string &tok : split_top(inner.substr(lb + 1, rb - lb - 1))) ci.push_back(operand_index(tok));
  if (mi < 0 || (int)ci.size() != dims) return false;
  std::vector<std::string> cons;
  for (const std::string &k : split_top(text.substr(c0 + 1, c1 - c0 - 1))) {
    if (starts_with(k, "=")) return false;  // an output would shift the operand numbers
    if (!starts_with(k, "~{")) cons.push_back(k);
  }
  const size_t p0 = text.find('(', c1), p1 = text.rfind(')');
  if (p0 == std::string::npos || p1 == std::string::npos || p1 <= p0) return false;
  const std::vector<std::string> args = split_top(text.substr(p0 + 1, p1 - p0 - 1));
  auto arg = [&](int k, std::string &ty, std::string &v) -> bool {
    if (k < 0 || k >= (int)args.size() || k >= (int)cons.size()) return false;
    const size_t sp = args[k].rfind(' ');
    if (sp == std::string::npos) return false;
    ty = trim(args[k].substr(0, sp));
    v = trim(args[k].substr(sp + 1));
    return !v.empty() && v[0] == '%';
  };
  TmaSite out;
  out.dims = dims;
  if (!arg(mi, out.tmap_type, out.tmap) || cons[mi] != "l") return false;
  if (!(starts_with(out.tmap_type, "ptr") || out.tmap_type == "i64")) return false;
  for (int k : ci) {
    std::string ty, v;
    if (!arg(k, ty, v) || ty != "i32" || cons[k] != "r") return false;
    out.coords.push_back(v);
  }
  out.text = text;
  s = out;
  return true;
}

void insert_after(Block &b, int idx, const std::vector<Inst> &code) {
  b.insts.insert(b.insts.begin() + idx + 1, code.begin(), code.end());
}
void insert_before(Block &b, int idx, const std::vector<Inst> &code) {
  b.insts.insert(b.insts.begin() + idx, code.begin(), code.end());
}

// Replace uses of `from` by `to` wherever `to` (defined in block `blk` at
// index `after`) dominates the use, within loop L: the rest of block `blk`,
// the non-phi instructions of the loop blocks that `blk` dominates, and phi
// incoming values on edges leaving a block that `blk` dominates (the back
// edge into the header among them).
void replace_dominated(Function &f, int blk, int after, const Loop &L, const std::string &from,
                       const std::string &to) {
  const Cfg g(f);
  for (size_t i = after + 1; i < f.blocks[blk].insts.size(); ++i)
    if (f.blocks[blk].insts[i].opcode != "phi") replace_uses(f.blocks[blk].insts[i], from, to);
  auto edge_ok = [&](const std::string &pred_label) { return g.dominates(blk, f.block_index(pred_label)); };
  for (int b = 0; b < (int)f.blocks.size(); ++b) {
    if (!L.contains(b)) continue;
    const bool dom = b != blk && g.dominates(blk, b);
    for (Inst &in : f.blocks[b].insts) {
      if (in.opcode == "phi")
        rewrite_phi_incoming(in, from, to, edge_ok);
      else if (dom)
        replace_uses(in, from, to);
    }
  }
}

class Weaver {
 public:
  Weaver(Module &m, Function &f, const Config &c, Notes &n) : m(m), f(f), c(c), n(n) {}

  bool run() {
    const bool body = f.header.find(kTaskBody) != std::string::npos;
    Defs defs(f);
    // ---- phase 0: detection while the function is untouched
    std::vector<Loop> loops = find_loops(f);
    std::vector<Site> sites;
    async_sites.clear();
    tma_sites.clear();
    if (c.policy || c.shed) {
      const std::set<std::string> written = written_roots(f, defs);
      for (size_t li = 0; li < loops.size(); ++li) {
        const Loop &L = loops[li];
        for (int b = 0; b < (int)f.blocks.size(); ++b)
          for (size_t i = 0; L.contains(b) && i < f.blocks[b].insts.size(); ++i) {
            const Inst &in = f.blocks[b].insts[i];
            if (in.opcode != "load" || in.operands.empty()) continue;
            Mu mu = L.iv.empty() ? Mu::None : address_kind(f, defs, L, in.operands.back());
            if (mu == Mu::None) continue;
            if (written.count(pointer_root(f, defs, in.operands.back()))) continue;  // not read-only
            Site s{b, (int)i, in.result, in.operands.back(), "", in.type, mu, (int)li};
            std::string t = in.text;
            size_t comma = t.find(',');
            s.ptr_type = trim(t.substr(comma + 1));
            s.ptr_type = s.ptr_type.substr(0, s.ptr_type.find(s.ptr) - 1);
            s.ptr_type = trim(s.ptr_type);
            sites.push_back(s);
            if (sites.size() >= 4) break;
          }
      }
      if (c.policy)
        for (size_t li = 0; li < loops.size(); ++li) {
          const Loop &L = loops[li];
          if (L.iv.empty()) continue;
          for (int b = 0; b < (int)f.blocks.size(); ++b)
            for (const Inst &in : f.blocks[b].insts) {
              if (!L.contains(b)) break;
              AsyncSite as;
              if (in.opcode != "call" || !parse_cp_async(in.text, as.src, as.src_type)) continue;
              if (address_kind(f, defs, L, as.src) == Mu::None) continue;
              as.text = in.text;
              as.loop = (int)li;
              if (async_sites.size() < 4) async_sites.push_back(as);
            }
        }
      if (c.policy)
        for (size_t li = 0; li < loops.size(); ++li) {
          const Loop &L = loops[li];
          if (L.iv.empty()) continue;
          for (int b = 0; b < (int)f.blocks.size(); ++b)
            for (const Inst &in : f.blocks[b].insts) {
              if (!L.contains(b)) break;
              TmaSite ts;
              if (in.opcode != "call" || !parse_tma_load(in.text, ts)) continue;
              ts.loop = (int)li;
              if (tma_sites.size() < 4) tma_sites.push_back(ts);
            }
        }
      for (const Loop &L : loops)
        if (L.iv.empty()) n.add(f.name + ": loop at block " + std::to_string(L.header) +
                                " has no canonical induction variable: shed/prefetch declined there");
    }
    std::vector<std::string> old_pid;
    const std::string slot_sreg = std::string("ctaid.") + "xyz"[c.slot_axis];
    const std::string slot_fn = "@llvm.nvvm.read.ptx.sreg." + slot_sreg;
    if (!body)
      for (Block &b : f.blocks)
        for (Inst &in : b.insts)
          if (in.opcode == "call" && in.text.find(slot_fn + "()") != std::string::npos && !in.result.empty())
            old_pid.push_back(in.result);

    // ---- phase 1: entry code
    std::vector<Inst> entry;
    Slot ctrl = load_slot(f, entry, m, c, "@__sched_ctrl", c.bake_ctrl);
    std::string zero = zero_table(m);
    std::string ctrl_ptr = zero, ctrl_armed = "false";
    if (ctrl.available) {
      ctrl_ptr = f.unique("%sched.ctrl");
      entry.push_back(I("  " + ctrl_ptr + " = select i1 " + ctrl.armed + ", ptr " + ctrl.ptr + ", ptr " + zero));
      ctrl_armed = ctrl.armed;
    }
    Slot timer = c.timer ? load_slot(f, entry, m, c, "@__sched_timer", c.bake_timer) : Slot();
    std::string t0, timer_gate;
    if (timer.available) {
      declare_sreg(m, "clock64");
      t0 = f.unique("%sched.t0");
      entry.push_back(I("  " + t0 + " = call i64 @llvm.nvvm.read.ptx.sreg.clock64()"));
      std::string fp = f.unique("%sched.flags.p"), fl = f.unique("%sched.flags"), bit = f.unique("%sched.flags.bit");
      std::string off = f.unique("%sched.timer.off");
      timer_gate = f.unique("%sched.timer.gate");
      entry.push_back(I("  " + fp + " = getelementptr i8, ptr " + ctrl_ptr + ", i64 24"));
      entry.push_back(I("  " + fl + " = load i32, ptr " + fp + ", align 4"));
      entry.push_back(I("  " + bit + " = and i32 " + fl + ", 1"));
      entry.push_back(I("  " + off + " = icmp ne i32 " + bit + ", 0"));
      entry.push_back(I("  " + timer_gate + " = select i1 " + ctrl_armed + ", i1 " + off + ", i1 false"));
    }
    std::string task;
    if (body) {
      task = f.param_names.back();
    } else {
      declare_sreg(m, slot_sreg);
      std::string pid = f.unique("%sched.pid");
      entry.push_back(I("  " + pid + " = call i32 " + slot_fn + "()"));
      task = pid;
      Slot order = c.pi ? load_slot(f, entry, m, c, "@__sched_task_order", c.bake_order) : Slot();
      if (order.available) task = emit_remap(entry, order, pid, ctrl_ptr, slot_sreg);
      if (order.available && !old_pid.empty())
        n.add(f.name + ": remapped " + std::to_string(old_pid.size()) + " ctaid use(s) through task_order");
    }
    // policy flags / shed budget from the task's row
    std::string urgent, polite, budget;
    bool need_row = (!sites.empty() || !async_sites.empty() || !tma_sites.empty()) && ctrl.available;
    std::string row;
    if (need_row) {
      std::string inb = f.unique("%sched.row.inb"), use = f.unique("%sched.row.use"), idx = f.unique("%sched.row.idx");
      std::string idx64 = f.unique("%sched.row.idx64"), off = f.unique("%sched.row.off");
      row = f.unique("%sched.row");
      entry.push_back(I("  " + inb + " = icmp ult i32 " + task + ", " + std::to_string(c.max_tasks)));
      entry.push_back(I("  " + use + " = and i1 " + ctrl_armed + ", " + inb));
      entry.push_back(I("  " + idx + " = select i1 " + use + ", i32 " + task + ", i32 0"));
      entry.push_back(I("  " + idx64 + " = zext i32 " + idx + " to i64"));
      entry.push_back(I("  " + off + " = mul i64 " + idx64 + ", 8"));
      std::string r0 = f.unique("%sched.row.base");
      entry.push_back(I("  " + r0 + " = getelementptr i8, ptr " + ctrl_ptr + ", i64 32"));
      entry.push_back(I("  " + row + " = getelementptr i8, ptr " + r0 + ", i64 " + off));
    }
    if (need_row && c.policy) {
      std::string qv = f.unique("%sched.q"), hp = f.unique("%sched.hint.p"), hint = f.unique("%sched.hint");
      std::string lp = f.unique("%sched.lambda.p"), lam = f.unique("%sched.lambda.bw");
      std::string a1 = f.unique("%sched.score.qdt"), a2 = f.unique("%sched.score.ldr"), a3 = f.unique("%sched.score.x");
      std::string score = f.unique("%sched.score"), ok = f.unique("%sched.score.ok");
      std::string ha = f.unique("%sched.hint.auto"), hu = f.unique("%sched.hint.urgent"), hpo = f.unique("%sched.hint.polite");
      std::string au = f.unique("%sched.auto.urgent");
      urgent = f.unique("%sched.urgent");
      polite = hpo;
      entry.push_back(I("  " + qv + " = load float, ptr " + row + ", align 4"));
      entry.push_back(I("  " + hp + " = getelementptr i8, ptr " + row + ", i64 6"));
      entry.push_back(I("  " + hint + " = load i8, ptr " + hp + ", align 1"));
      entry.push_back(I("  " + lp + " = getelementptr i8, ptr " + ctrl_ptr + ", i64 8"));
      entry.push_back(I("  " + lam + " = load float, ptr " + lp + ", align 4"));
      entry.push_back(I("  " + a1 + " = fmul float " + qv + ", " + fmt_double((float)c.dT)));
      entry.push_back(I("  " + a2 + " = fmul float " + lam + ", " + fmt_double((float)c.dR)));
      entry.push_back(I("  " + a3 + " = fsub float " + a1 + ", " + a2));
      entry.push_back(I("  " + score + " = fsub float " + a3 + ", " + fmt_double((float)c.H)));
      entry.push_back(I("  " + ok + " = fcmp ogt float " + score + ", 0.000000e+00"));
      entry.push_back(I("  " + ha + " = icmp eq i8 " + hint + ", 0"));
      entry.push_back(I("  " + hu + " = icmp eq i8 " + hint + ", 1"));
      entry.push_back(I("  " + hpo + " = icmp eq i8 " + hint + ", 2"));
      entry.push_back(I("  " + au + " = and i1 " + ha + ", " + ok));
      entry.push_back(I("  " + urgent + " = or i1 " + hu + ", " + au));
    }
    if (need_row && c.shed) {
      std::string tp = f.unique("%sched.tau.p"), t16 = f.unique("%sched.tau16"), tau = f.unique("%sched.tau");
      std::string none = f.unique("%sched.tau.none");
      budget = f.unique("%sched.budget");
      entry.push_back(I("  " + tp + " = getelementptr i8, ptr " + row + ", i64 4"));
      entry.push_back(I("  " + t16 + " = load i16, ptr " + tp + ", align 2"));
      entry.push_back(I("  " + tau + " = zext i16 " + t16 + " to i32"));
      entry.push_back(I("  " + none + " = icmp eq i32 " + tau + ", 0"));
      entry.push_back(I("  " + budget + " = select i1 " + none + ", i32 -1, i32 " + tau));
    }
    const bool pdl = c.pdl && !body && sm() >= 90;
    if (pdl) entry.push_back(I("  call void asm sideeffect \"griddepcontrol.wait;\", \"~{memory}\"()"));

    // place entry code after the entry block's allocas
    Block &eb = f.blocks[0];
    size_t ip = 0;
    while (ip < eb.insts.size() && eb.insts[ip].opcode == "alloca") ++ip;
    eb.insts.insert(eb.insts.begin() + ip, entry.begin(), entry.end());

    // old ctaid reads -> task
    if (!body && task != "" && !old_pid.empty()) {
      for (Block &b : f.blocks) {
        for (auto it = b.insts.begin(); it != b.insts.end();) {
          bool old = std::find(old_pid.begin(), old_pid.end(), it->result) != old_pid.end();
          if (old) {
            it = b.insts.erase(it);
            continue;
          }
          ++it;
        }
        for (Inst &in : b.insts)
          for (const std::string &o : old_pid) replace_uses(in, o, task);
      }
    }

    // ---- phase 2: body (shed first: it needs the block layout of detection)
    if (!budget.empty() && c.shed) emit_shed(sites, loops, budget);
    if (!urgent.empty() && c.policy) emit_policy(sites, loops, urgent, polite);
    if (timer.available) emit_timer(timer, t0, timer_gate, task);
    if (pdl) {
      for (Block &b : f.blocks)
        for (size_t i = 0; i < b.insts.size(); ++i)
          if (b.insts[i].opcode == "ret") {
            insert_before(b, (int)i, {I("  call void asm sideeffect \"griddepcontrol.launch_dependents;\", \"~{memory}\"()")});
            ++i;
          }
      n.add(f.name + ": PDL overlap points woven");
    }
    mark();
    return true;
  }

 private:
  Module &m;
  Function &f;
  const Config &c;
  Notes &n;
  std::vector<AsyncSite> async_sites;
  std::vector<TmaSite> tma_sites;

  int sm() const {
    if (starts_with(m.target_cpu, "sm_")) return std::atoi(m.target_cpu.c_str() + 3);
    return 100;  // this framework targets sm_100a
  }

  void mark() {
    if (f.header.find(kInstrumented) == std::string::npos) {
      size_t brace = f.header.rfind('{');
      f.header = f.header.substr(0, brace) + kInstrumented + " {";
    }
  }

  std::string emit_remap(std::vector<Inst> &e, const Slot &order, const std::string &pid,
                         const std::string &ctrl, const std::string &slot_sreg) {
    declare_sreg(m, "n" + slot_sreg);
    std::string zero = zero_table(m);
    std::string nt = f.unique("%sched.ntiles");
    e.push_back(I("  " + nt + " = call i32 @llvm.nvvm.read.ptx.sreg.n" + slot_sreg + "()"));
    std::string inb = f.unique("%sched.pid.inb"), use = f.unique("%sched.order.use");
    e.push_back(I("  " + inb + " = icmp ult i32 " + pid + ", " + std::to_string(c.max_tasks)));
    e.push_back(I("  " + use + " = and i1 " + order.armed + ", " + inb));
    std::string table = order.ptr;
    std::string chan_ok;
    if (c.order_indirect) {
      // the slot word holds a pointer to the device order table; 0 = identity
      std::string chan = f.unique("%sched.order.chan"), sb = f.unique("%sched.order.slotp");
      e.push_back(I("  " + sb + " = select i1 " + order.armed + ", ptr " + order.ptr + ", ptr " + zero));
      e.push_back(I("  " + chan + " = load ptr, ptr " + sb + ", align 8"));
      chan_ok = f.unique("%sched.order.chan.armed");
      e.push_back(I("  " + chan_ok + " = icmp ne ptr " + chan + ", null"));
      std::string u2 = f.unique("%sched.order.use2");
      e.push_back(I("  " + u2 + " = and i1 " + use + ", " + chan_ok));
      use = u2;
      table = chan;
    }
    std::string base = f.unique("%sched.order.base"), idx = f.unique("%sched.order.idx");
    std::string gep = f.unique("%sched.order.gep"), mapped = f.unique("%sched.task.mapped");
    e.push_back(I("  " + base + " = select i1 " + use + ", ptr " + table + ", ptr " + zero));
    e.push_back(I("  " + idx + " = select i1 " + use + ", i32 " + pid + ", i32 0"));
    e.push_back(I("  " + gep + " = getelementptr i32, ptr " + base + ", i32 " + idx));
    e.push_back(I("  " + mapped + " = load i32, ptr " + gep + ", align 4"));
    // whole-launch validity: order_size == 0 (unchecked) or == launch size
    std::string osp = f.unique("%sched.order.size.p"), osz = f.unique("%sched.order.size");
    std::string unchk = f.unique("%sched.order.unchecked"), match = f.unique("%sched.order.match");
    std::string valid = f.unique("%sched.order.valid"), szok = f.unique("%sched.order.szok");
    e.push_back(I("  " + osp + " = getelementptr i8, ptr " + ctrl + ", i64 28"));
    e.push_back(I("  " + osz + " = load i32, ptr " + osp + ", align 4"));
    e.push_back(I("  " + unchk + " = icmp eq i32 " + osz + ", 0"));
    e.push_back(I("  " + match + " = icmp eq i32 " + osz + ", " + nt));
    e.push_back(I("  " + valid + " = or i1 " + unchk + ", " + match));
    e.push_back(I("  " + szok + " = and i1 " + valid + ", " + use));
    // per-launch bound: an entry outside the grid falls back to pid
    std::string ingrid = f.unique("%sched.task.ingrid"), ok = f.unique("%sched.task.ok");
    std::string task = f.unique("%sched.task");
    e.push_back(I("  " + ingrid + " = icmp ult i32 " + mapped + ", " + nt));
    e.push_back(I("  " + ok + " = and i1 " + ingrid + ", " + szok));
    e.push_back(I("  " + task + " = select i1 " + ok + ", i32 " + mapped + ", i32 " + pid));
    return task;
  }

  // shed: score -> -inf (softmax) or value -> 0 (linear) beyond the budget
  void emit_shed(const std::vector<Site> &sites, const std::vector<Loop> &loops, const std::string &budget) {
    bool softmax = false;
    for (const Site &s : sites)
      if (!find_softmax_score(f, s.load).empty()) softmax = true;
    std::map<int, std::string> ctr_of_loop;
    // process sites bottom-up so earlier insertions do not shift later indices
    std::vector<Site> order(sites.begin(), sites.end());
    std::sort(order.begin(), order.end(), [](const Site &a, const Site &b) {
      return a.block != b.block ? a.block > b.block : a.inst > b.inst;
    });
    // resolve every site's mask target before editing (a mask's select would
    // otherwise look like a new score to the next site)
    std::vector<std::pair<std::string, std::string>> targets;  // (target, score)
    {
      std::set<std::string> seen;
      for (const Site &s : order) {
        std::string sc = find_softmax_score(f, s.load);
        if (softmax && sc.empty()) continue;  // V-like load: its weight is already masked
        std::string tg = sc.empty() ? s.load : sc;
        if (seen.insert(tg).second) targets.push_back({tg, sc});
      }
    }
    for (const auto &tgt : targets) {
      const std::string score0 = tgt.second;
      const std::string target0 = tgt.first;
      int li = -1;
      {
        Defs d0(f);
        auto it0 = d0.at.find(target0);
        if (it0 == d0.at.end()) continue;
        int tb = it0->second.first;
        for (size_t k = 0; k < loops.size(); ++k) {
          const Loop &Lk = loops[k];
          if (Lk.iv.empty() || !in_loop(Lk, tb)) continue;
          if (li < 0 || Lk.size < loops[li].size) li = (int)k;  // innermost loop around the site
        }
      }
      if (li < 0) {
        n.add(f.name + ": shed declined -- no loop with a canonical induction variable around the site");
        continue;
      }
      const Loop &L = loops[li];
      const int s_loop = li;
      std::string ctr = L.iv;
      if (int_bits(L.iv_type) != 32 && ctr_of_loop.find(s_loop) == ctr_of_loop.end()) {
        std::string t = f.unique("%sched.shed.ctr");
        Block &h = f.blocks[L.header];
        size_t p = 0;
        while (p < h.insts.size() && h.insts[p].opcode == "phi") ++p;
        h.insts.insert(h.insts.begin() + p,
                       I("  " + t + " = " + (int_bits(L.iv_type) > 32 ? "trunc " : "zext ") + L.iv_type + " " + L.iv + " to i32"));
        ctr_of_loop[s_loop] = t;
      }
      if (ctr_of_loop.count(s_loop)) ctr = ctr_of_loop[s_loop];
      // locate the target again (the header insert may have shifted it)
      Defs defs(f);
      const std::string &score = score0;
      const std::string &target = target0;
      auto it = defs.at.find(target);
      if (it == defs.at.end()) continue;
      int b = it->second.first, i = it->second.second;
      const Inst &def = f.blocks[b].insts[i];
      if (!is_float_ty(def.type)) continue;
      if (!in_loop(L, b)) {
        n.add(f.name + ": shed declined -- score outside the loop body");
        continue;
      }
      std::string keep = f.unique("%sched.keep");
      std::string sel = f.unique(score.empty() ? "%sched.shed.val" : "%sched.shed.score");
      std::string fill = score.empty() ? "0.000000e+00" : kNegInf;
      insert_after(f.blocks[b], i, {I("  " + keep + " = icmp ult i32 " + ctr + ", " + budget),
                                     I("  " + sel + " = select i1 " + keep + ", " + def.type + " " + target + ", " + def.type + " " + fill)});
      replace_dominated(f, b, i + 2, L, target, sel);
      n.add(f.name + (score.empty() ? ": shed linear value mask woven (->0)" : ": shed softmax score mask woven (-inf)"));
    }
  }

  // policy: urgent -> prefetch.global.L2::evict_last ahead (affine streams),
  // polite -> discard the consumed L2 line; both predicated inline asm.
  void emit_policy(const std::vector<Site> &sites, const std::vector<Loop> &loops, const std::string &urgent,
                   const std::string &polite) {
    if (sm() < 80) return;
    std::string ui = f.unique("%sched.urgent.i32"), pi = f.unique("%sched.polite.i32");
    {
      Block &eb = f.blocks[0];
      size_t p = 0;
      for (size_t k = 0; k < eb.insts.size(); ++k)
        if (eb.insts[k].result == urgent || eb.insts[k].result == polite) p = k + 1;
      insert_after(eb, (int)p - 1, {I("  " + ui + " = zext i1 " + urgent + " to i32"), I("  " + pi + " = zext i1 " + polite + " to i32")});
    }
    for (const Site &s0 : sites) {
      Defs defs(f);
      auto it = defs.at.find(s0.load);
      if (it == defs.at.end()) continue;
      int b = it->second.first, i = it->second.second;
      const Loop &L = loops[s0.loop];
      std::vector<Inst> before, after;
      std::string pint = f.unique("%sched.pf.int");
      before.push_back(I("  " + pint + " = ptrtoint " + s0.ptr_type + " " + s0.ptr + " to i64"));
      long long step = 0;
      const Inst *gep = defs.get(f, s0.ptr);
      bool affine = false;
      int elem = 0;
      if (gep && gep->opcode == "getelementptr" && s0.mu == Mu::Arith) {
        std::string t = gep->text.substr(gep->text.find("getelementptr") + 13);
        std::vector<std::string> w;
        std::string ty = trim(t);
        while (starts_with(ty, "inbounds ") || starts_with(ty, "nuw ") || starts_with(ty, "nusw ")) ty = trim(ty.substr(ty.find(' ')));
        std::string et = trim(ty.substr(0, ty.find(',')));
        elem = type_bytes(et);
        if (elem > 0 && gep->operands.size() == 2 && iv_step(f, defs, L.iv, gep->operands[1], step)) affine = step != 0;
      }
      if (affine) {
        std::string ahead = f.unique("%sched.pf.ahead");
        before.push_back(I("  " + ahead + " = add i64 " + pint + ", " + std::to_string(step * elem * (long long)c.prefetch_dist)));
        before.push_back(I("  call void asm sideeffect \"{ .reg .pred p; setp.ne.u32 p, $1, 0; @p prefetch.global.L2::evict_last [$0]; }\", \"l,r,~{memory}\"(i64 " +
                           ahead + ", i32 " + ui + ")"));
      } else {
        n.add(f.name + ": prefetch-ahead declined on an index-based stream (no affine step); polite tier only");
      }
      std::string al = f.unique("%sched.dc.line");
      after.push_back(I("  " + al + " = and i64 " + pint + ", -128"));
      // polite: demote the consumed line to normal eviction priority. (An L2
      // discard would invalidate the line without write-back: data written by
      // a recent kernel and still dirty in L2 -- KV appended one step ago --
      // would be lost, so it is not result-invariant and is never emitted.)
      after.push_back(I("  call void asm sideeffect \"{ .reg .pred p; setp.ne.u32 p, $1, 0; @p applypriority.global.L2::evict_normal [$0], 128; }\", \"l,r,~{memory}\"(i64 " +
                        al + ", i32 " + pi + ")"));
      insert_after(f.blocks[b], i, after);
      insert_before(f.blocks[b], i, before);
      n.add(f.name + ": L2 policy woven at a stream load");
    }
    for (const AsyncSite &as : async_sites) emit_async_warm(as, loops[as.loop], ui);
    for (const TmaSite &ts : tma_sites) emit_tma_warm(ts, loops[ts.loop], ui);
  }

  // TMA stream warming: the same box `dist` iterations ahead, prefetched into
  // L2 by the urgent tier (cp.async.bulk.prefetch.tensor, sm_90 and later)
  // right before the load. Coordinates that do not move with the IV are
  // kept; an advanced coordinate past the tensor's extent is a prefetch of
  // nothing. The innermost coordinate moves by a multiple of its own
  // per-iteration step, so its 16-byte alignment is the load's.
  void emit_tma_warm(const TmaSite &ts, const Loop &L, const std::string &ui) {
    if (sm() < 90) {
      n.add(f.name + ": TMA stream warming needs sm_90 or later; declined");
      return;
    }
    for (Block &b : f.blocks)
      for (size_t i = 0; i < b.insts.size(); ++i) {
        if (b.insts[i].text != ts.text) continue;
        Defs defs(f);
        std::vector<Inst> code;
        std::vector<std::string> ahead = ts.coords;
        bool moves = false;
        for (size_t j = 0; j < ts.coords.size(); ++j) {
          long long step = 0;
          if (!iv_step(f, defs, L.iv, ts.coords[j], step)) {
            n.add(f.name + ": TMA stream warming declined (a coordinate is not affine in the IV)");
            return;
          }
          if (step == 0) continue;
          moves = true;
          ahead[j] = f.unique("%sched.tpf.c");
          code.push_back(I("  " + ahead[j] + " = add i32 " + ts.coords[j] + ", " +
                           std::to_string(step * (long long)c.prefetch_dist)));
        }
        if (!moves) {
          n.add(f.name + ": TMA stream warming declined (no coordinate advances with the loop)");
          return;
        }
        const int D = ts.dims;
        std::string tmpl = "{ .reg .pred p; setp.ne.u32 p, $" + std::to_string(D + 1) +
                           ", 0; @p cp.async.bulk.prefetch.tensor." + std::to_string(D) + "d.L2.global.tile [$0, {";
        std::string cons = "l", args = ts.tmap_type + " " + ts.tmap;
        for (int j = 0; j < D; ++j) {
          tmpl += (j ? ", $" : "$") + std::to_string(j + 1);
          cons += ",r";
          args += ", i32 " + ahead[j];
        }
        tmpl += "}]; }";
        cons += ",r,~{memory}";
        args += ", i32 " + ui;
        code.push_back(I("  call void asm sideeffect \"" + tmpl + "\", \"" + cons + "\"(" + args + ")"));
        insert_before(b, (int)i, code);
        n.add(f.name + ": TMA stream warming woven (urgent tensor prefetch ahead)");
        return;
      }
    n.add(f.name + ": TMA load moved; warming skipped");
  }

  // cp.async source warming: prefetch the source `dist` iterations ahead,
  // predicated on the urgent tier, when the source is affine in the IV.
  void emit_async_warm(const AsyncSite &as, const Loop &L, const std::string &ui) {
    for (Block &b : f.blocks)
      for (size_t i = 0; i < b.insts.size(); ++i) {
        if (b.insts[i].text != as.text) continue;
        Defs defs(f);
        const Inst *gep = defs.get(f, as.src);
        long long step = 0;
        int elem = 0;
        if (gep && gep->opcode == "getelementptr" && gep->operands.size() == 2) {
          std::string ty = trim(gep->text.substr(gep->text.find("getelementptr") + 13));
          while (starts_with(ty, "inbounds ") || starts_with(ty, "nuw ") || starts_with(ty, "nusw "))
            ty = trim(ty.substr(ty.find(' ')));
          elem = type_bytes(trim(ty.substr(0, ty.find(','))));
          if (elem <= 0 || !iv_step(f, defs, L.iv, gep->operands[1], step)) step = 0;
        }
        if (step == 0) {
          n.add(f.name + ": cp.async source warming declined (no affine step)");
          return;
        }
        std::string pint = f.unique("%sched.apf.int"), ahead = f.unique("%sched.apf.ahead");
        insert_before(b, (int)i,
                      {I("  " + pint + " = ptrtoint " + as.src_type + " " + as.src + " to i64"),
                       I("  " + ahead + " = add i64 " + pint + ", " + std::to_string(step * elem * (long long)c.prefetch_dist)),
                       I("  call void asm sideeffect \"{ .reg .pred p; setp.ne.u32 p, $1, 0; @p prefetch.global.L2::evict_last [$0]; }\", \"l,r,~{memory}\"(i64 " +
                         ahead + ", i32 " + ui + ")")});
        n.add(f.name + ": cp.async source warming woven (urgent prefetch ahead)");
        return;
      }
    n.add(f.name + ": cp.async site moved; warming skipped");
  }

  void emit_timer(const Slot &timer, const std::string &t0, const std::string &gate, const std::string &task) {
    declare_sreg(m, "tid.x");
    declare_sreg(m, "tid.y");
    declare_sreg(m, "tid.z");
    size_t nb = f.blocks.size();
    for (size_t bi = 0; bi < nb; ++bi) {
      Block &b = f.blocks[bi];
      if (b.insts.empty() || b.insts.back().opcode != "ret") continue;
      Inst ret = b.insts.back();
      b.insts.pop_back();
      std::vector<Inst> e;
      std::string t1 = f.unique("%sched.t1"), cyc = f.unique("%sched.cycles");
      e.push_back(I("  " + t1 + " = call i64 @llvm.nvvm.read.ptx.sreg.clock64()"));
      e.push_back(I("  " + cyc + " = sub i64 " + t1 + ", " + t0));
      std::string tx = f.unique("%sched.tid.x"), ty = f.unique("%sched.tid.y"), tz = f.unique("%sched.tid.z");
      std::string o1 = f.unique("%sched.tid.or"), o2 = f.unique("%sched.tid.or"), tzero = f.unique("%sched.tid.zero");
      e.push_back(I("  " + tx + " = call i32 @llvm.nvvm.read.ptx.sreg.tid.x()"));
      e.push_back(I("  " + ty + " = call i32 @llvm.nvvm.read.ptx.sreg.tid.y()"));
      e.push_back(I("  " + tz + " = call i32 @llvm.nvvm.read.ptx.sreg.tid.z()"));
      e.push_back(I("  " + o1 + " = or i32 " + tx + ", " + ty));
      e.push_back(I("  " + o2 + " = or i32 " + o1 + ", " + tz));
      e.push_back(I("  " + tzero + " = icmp eq i32 " + o2 + ", 0"));
      std::string inb = f.unique("%sched.timer.inb"), on = f.unique("%sched.timer.on");
      std::string a1 = f.unique("%sched.timer.a"), a2 = f.unique("%sched.timer.b"), ok = f.unique("%sched.timer.ok");
      e.push_back(I("  " + inb + " = icmp ult i32 " + task + ", " + std::to_string(c.max_tasks)));
      e.push_back(I("  " + on + " = xor i1 " + gate + ", true"));
      e.push_back(I("  " + a1 + " = and i1 " + tzero + ", " + timer.armed));
      e.push_back(I("  " + a2 + " = and i1 " + a1 + ", " + inb));
      e.push_back(I("  " + ok + " = and i1 " + a2 + ", " + on));
      std::string lab_do = f.unique("%sched.timer.do").substr(1), lab_ret = f.unique("%sched.timer.ret").substr(1);
      e.push_back(I("  br i1 " + ok + ", label %" + lab_do + ", label %" + lab_ret));
      b.insts.insert(b.insts.end(), e.begin(), e.end());
      Block bdo;
      bdo.label = lab_do;
      std::string rows = timer.ptr;
      std::vector<Inst> d;
      if (c.timer_indirect) {
        // the slot word holds the row-table address; 0 = timer off
        std::string chan = f.unique("%sched.timer.chan"), chok = f.unique("%sched.timer.chan.armed");
        d.push_back(I("  " + chan + " = load ptr, ptr " + timer.ptr + ", align 8"));
        d.push_back(I("  " + chok + " = icmp ne ptr " + chan + ", null"));
        std::string lab_w = f.unique("%sched.timer.write").substr(1);
        d.push_back(I("  br i1 " + chok + ", label %" + lab_w + ", label %" + lab_ret));
        bdo.insts = d;
        f.blocks.push_back(bdo);
        bdo = Block();
        bdo.label = lab_w;
        d.clear();
        rows = chan;
      }
      std::string slot = f.unique("%sched.timer.row"), old = f.unique("%sched.timer.old");
      d.push_back(I("  " + slot + " = getelementptr i64, ptr " + rows + ", i32 " + task));
      d.push_back(I("  " + old + " = atomicrmw add ptr " + slot + ", i64 " + cyc + " monotonic, align 8"));
      d.push_back(I("  br label %" + lab_ret));
      bdo.insts = d;
      f.blocks.push_back(bdo);
      Block br;
      br.label = lab_ret;
      br.insts.push_back(ret);
      f.blocks.push_back(br);
    }
  }
};

}  // namespace

bool run_weave(Module &m, const Config &c, Notes &notes) {
  bool changed = false;
  for (Function &f : m.functions) {
    const bool body = f.header.find(kTaskBody) != std::string::npos;
    if (!body && !f.is_kernel) continue;
    if (f.header.find(kWqDriver) != std::string::npos || f.header.find(kInstrumented) != std::string::npos) continue;
    notes.add("weaving " + f.name + (body ? " (task body)" : " (kernel)"));
    changed |= Weaver(m, f, c, notes).run();
  }
  return changed;
}

}  // namespace weave
