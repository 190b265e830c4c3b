// cfg.cpp -- control-flow analysis over the weaver's IR model (see cfg.h).
#include "cfg.h"

#include <algorithm>
#include <cctype>
#include <functional>

namespace weave {

namespace {

bool label_char(char c) {
  return std::isalnum(static_cast<unsigned char>(c)) || c == '.' || c == '_' || c == '-' || c == '$';
}

// The add that steps an IV by one: `%n = add [flags] <ty> %iv, 1` or `1, %iv`.
bool is_unit_step(const Inst &d, const std::string &iv) {
  if (d.opcode != "add") return false;
  std::string t = trim(d.text);
  size_t eq = t.find('=');
  if (eq == std::string::npos) return false;
  std::string rest = trim(t.substr(eq + 1));
  rest = trim(rest.substr(3));  // "add"
  // drop wrap flags, then the type
  for (;;) {
    if (starts_with(rest, "nuw ") || starts_with(rest, "nsw ")) {
      rest = trim(rest.substr(4));
      continue;
    }
    break;
  }
  size_t sp = rest.find(' ');
  if (sp == std::string::npos) return false;
  rest = trim(rest.substr(sp + 1));
  size_t comma = rest.find(',');
  if (comma == std::string::npos) return false;
  const std::string a = trim(rest.substr(0, comma)), b = trim(rest.substr(comma + 1));
  return (a == iv && b == "1") || (a == "1" && b == iv);
}

const Inst *definition(const Function &f, const std::string &v) {
  for (const Block &b : f.blocks)
    for (const Inst &in : b.insts)
      if (in.result == v) return &in;
  return nullptr;
}

}  // namespace

std::vector<std::string> branch_labels(const std::string &text) {
  std::vector<std::string> out;
  const std::string key = "label %";
  for (size_t p = text.find(key); p != std::string::npos; p = text.find(key, p + 1)) {
    size_t s = p + key.size(), e = s;
    if (e < text.size() && text[e] == '"') {  // quoted name
      size_t close = text.find('"', e + 1);
      if (close == std::string::npos) break;
      out.push_back(text.substr(e + 1, close - e - 1));
      continue;
    }
    while (e < text.size() && label_char(text[e])) ++e;
    if (e > s) out.push_back(text.substr(s, e - s));
  }
  return out;
}

std::vector<std::pair<std::string, std::string>> phi_incoming(const std::string &phi_text) {
  std::vector<std::pair<std::string, std::string>> out;
  size_t p = phi_text.find('[');
  while (p != std::string::npos) {
    size_t q = phi_text.find(']', p);
    if (q == std::string::npos) break;
    std::string inner = phi_text.substr(p + 1, q - p - 1);
    size_t comma = inner.rfind(',');
    if (comma != std::string::npos) {
      std::string val = trim(inner.substr(0, comma));
      std::string lab = trim(inner.substr(comma + 1));
      if (!lab.empty() && lab[0] == '%') lab = lab.substr(1);
      out.push_back({val, lab});
    }
    p = phi_text.find('[', q);
  }
  return out;
}

Cfg::Cfg(const Function &f) {
  const int n = (int)f.blocks.size();
  succ.assign(n, {});
  pred.assign(n, {});
  for (int b = 0; b < n; ++b) {
    const std::vector<Inst> &insts = f.blocks[b].insts;
    size_t t = 0;
    while (t < insts.size() && !insts[t].is_terminator()) ++t;
    for (size_t i = t; i < insts.size(); ++i)  // the terminator and any continuation lines
      for (const std::string &lab : branch_labels(insts[i].text)) {
        const int s = f.block_index(lab);
        if (s >= 0 && std::find(succ[b].begin(), succ[b].end(), s) == succ[b].end()) succ[b].push_back(s);
      }
    for (int s : succ[b]) pred[s].push_back(b);
  }
  // reverse postorder by an explicit DFS from the entry
  rpo_index.assign(n, -1);
  idom.assign(n, -1);
  if (n == 0) return;
  std::vector<int> post;
  std::vector<char> seen(n, 0);
  std::vector<std::pair<int, size_t>> stack{{0, 0}};
  seen[0] = 1;
  while (!stack.empty()) {
    auto &top = stack.back();
    if (top.second < succ[top.first].size()) {
      const int s = succ[top.first][top.second++];
      if (!seen[s]) {
        seen[s] = 1;
        stack.push_back({s, 0});
      }
    } else {
      post.push_back(top.first);
      stack.pop_back();
    }
  }
  rpo.assign(post.rbegin(), post.rend());
  for (size_t i = 0; i < rpo.size(); ++i) rpo_index[rpo[i]] = (int)i;
  // Cooper-Harvey-Kennedy: iterate idom to a fixed point in reverse postorder
  idom[0] = 0;
  auto intersect = [&](int a, int b) {
    while (a != b) {
      while (rpo_index[a] > rpo_index[b]) a = idom[a];
      while (rpo_index[b] > rpo_index[a]) b = idom[b];
    }
    return a;
  };
  for (bool changed = true; changed;) {
    changed = false;
    for (size_t i = 1; i < rpo.size(); ++i) {
      const int b = rpo[i];
      int d = -1;
      for (int p : pred[b]) {
        if (idom[p] < 0) continue;  // not processed yet (or unreachable)
        d = d < 0 ? p : intersect(p, d);
      }
      if (d >= 0 && idom[b] != d) {
        idom[b] = d;
        changed = true;
      }
    }
  }
}

bool Cfg::dominates(int a, int b) const {
  if (!reachable(a) || !reachable(b)) return false;
  for (int x = b;; x = idom[x]) {
    if (x == a) return true;
    if (x == idom[x]) return false;  // reached the entry
  }
}

void find_canonical_iv(const Function &f, NaturalLoop &L) {
  L.iv.clear();
  L.iv_type.clear();
  const Block &h = f.blocks[L.header];
  for (const Inst &in : h.insts) {
    if (in.opcode != "phi") break;
    if (in.type.size() < 2 || in.type[0] != 'i' || !std::isdigit(static_cast<unsigned char>(in.type[1]))) continue;
    bool ok = true, any_inside = false, any_outside = false;
    for (const auto &inc : phi_incoming(in.text)) {
      const int from = f.block_index(inc.second);
      if (L.contains(from)) {  // back edge: the value must step the phi by one
        const Inst *d = definition(f, inc.first);
        ok = ok && d != nullptr && is_unit_step(*d, in.result);
        any_inside = true;
      } else {  // entry edge: must start at zero
        ok = ok && inc.first == "0";
        any_outside = true;
      }
    }
    if (ok && any_inside && any_outside) {
      L.iv = in.result;
      L.iv_type = in.type;
      return;
    }
  }
}

std::vector<NaturalLoop> natural_loops(const Function &f, const Cfg &g) {
  const int n = (int)f.blocks.size();
  std::vector<NaturalLoop> loops;
  std::vector<int> loop_of_header(n, -1);
  for (int h : g.rpo) {  // headers in reverse postorder: an enclosing loop's header comes first
    for (int t : g.pred[h]) {
      if (!g.dominates(h, t)) continue;  // not a back edge
      int li = loop_of_header[h];
      if (li < 0) {
        li = loop_of_header[h] = (int)loops.size();
        NaturalLoop L;
        L.header = h;
        L.body.assign(n, 0);
        L.body[h] = 1;
        loops.push_back(L);
      }
      NaturalLoop &L = loops[li];
      L.latches.push_back(t);
      std::vector<int> work{t};
      while (!work.empty()) {
        const int b = work.back();
        work.pop_back();
        if (L.body[b]) continue;
        L.body[b] = 1;
        for (int p : g.pred[b])
          if (g.reachable(p)) work.push_back(p);
      }
    }
  }
  for (NaturalLoop &L : loops) {
    L.size = (int)std::count(L.body.begin(), L.body.end(), (char)1);
    find_canonical_iv(f, L);
  }
  return loops;
}

bool rewrite_phi_incoming(Inst &phi, const std::string &from, const std::string &to,
                          const std::function<bool(const std::string &)> &keep) {
  std::string t = phi.text, out;
  bool changed = false;
  size_t pos = 0;
  for (size_t p = t.find('[', pos); p != std::string::npos; p = t.find('[', pos)) {
    const size_t q = t.find(']', p);
    if (q == std::string::npos) break;
    out += t.substr(pos, p - pos);
    std::string inner = t.substr(p + 1, q - p - 1);
    const size_t comma = inner.rfind(',');
    if (comma != std::string::npos) {
      const std::string val = trim(inner.substr(0, comma));
      std::string lab = trim(inner.substr(comma + 1));
      const std::string bare = (!lab.empty() && lab[0] == '%') ? lab.substr(1) : lab;
      if (val == from && keep(bare)) {
        inner = " " + to + ", " + lab + " ";
        changed = true;
      }
    }
    out += "[" + inner + "]";
    pos = q + 1;
  }
  out += t.substr(pos);
  if (changed) phi = parse_inst(out);
  return changed;
}

}  // namespace weave
