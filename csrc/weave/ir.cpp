// ir.cpp -- parsing / printing of the textual IR model (see ir.h).
#include "ir.h"

#include <cctype>
#include <sstream>
#include <stdexcept>

namespace weave {

namespace {

bool name_char(char c) {
  return std::isalnum(static_cast<unsigned char>(c)) || c == '.' || c == '_' || c == '-' || c == '$';
}

const std::set<std::string> kFlags = {"nuw", "nsw", "exact", "fast", "nnan", "ninf", "nsz",
                                      "arcp", "contract", "afn", "reassoc", "disjoint", "nneg",
                                      "volatile", "atomic", "samesign"};
const std::set<std::string> kBinops = {"add", "sub", "mul", "fadd", "fsub", "fmul", "fdiv", "and",
                                       "or", "xor", "shl", "lshr", "ashr", "udiv", "sdiv", "urem",
                                       "srem", "frem", "fneg"};
const std::set<std::string> kCasts = {"zext", "sext", "trunc", "fptrunc", "fpext", "fptoui",
                                      "fptosi", "uitofp", "sitofp", "ptrtoint", "inttoptr",
                                      "bitcast", "addrspacecast"};

std::vector<std::string> words(const std::string &s) {
  std::vector<std::string> w;
  std::istringstream is(s);
  std::string x;
  while (is >> x) w.push_back(x);
  return w;
}

// A type token sequence at the start of `s` (handles "ptr addrspace(1)",
// "<4 x float>", "[4 x i32]", "{ i32, i32 }").
std::string leading_type(const std::string &s) {
  std::string t = trim(s);
  if (t.empty()) return "";
  char open = t[0];
  if (open == '<' || open == '[' || open == '{') {
    char close = open == '<' ? '>' : (open == '[' ? ']' : '}');
    int depth = 0;
    for (size_t i = 0; i < t.size(); ++i) {
      if (t[i] == open) ++depth;
      if (t[i] == close && --depth == 0) return t.substr(0, i + 1);
    }
    return t;
  }
  size_t e = 0;
  while (e < t.size() && !std::isspace(static_cast<unsigned char>(t[e])) && t[e] != ',') ++e;
  std::string ty = t.substr(0, e);
  std::string rest = trim(t.substr(e));
  if (ty == "ptr" && starts_with(rest, "addrspace(")) {
    size_t close = rest.find(')');
    ty += " " + rest.substr(0, close + 1);
  }
  return ty;
}

std::string strip_comment(const std::string &line) {
  bool in_str = false;
  for (size_t i = 0; i < line.size(); ++i) {
    if (line[i] == '"') in_str = !in_str;
    if (!in_str && line[i] == ';') return line.substr(0, i);
  }
  return line;
}

}  // namespace

std::string trim(const std::string &s) {
  size_t b = 0, e = s.size();
  while (b < e && std::isspace(static_cast<unsigned char>(s[b]))) ++b;
  while (e > b && std::isspace(static_cast<unsigned char>(s[e - 1]))) --e;
  return s.substr(b, e - b);
}

bool starts_with(const std::string &s, const std::string &p) {
  return s.size() >= p.size() && s.compare(0, p.size(), p) == 0;
}

// %-value names outside string literals, in order.
std::vector<std::string> value_tokens(const std::string &s) {
  std::vector<std::string> out;
  bool in_str = false;
  for (size_t i = 0; i < s.size(); ++i) {
    if (s[i] == '"') {
      in_str = !in_str;
      continue;
    }
    if (in_str || s[i] != '%') continue;
    if (i > 0 && name_char(s[i - 1])) continue;
    size_t j = i + 1;
    while (j < s.size() && name_char(s[j])) ++j;
    if (j > i + 1) out.push_back(s.substr(i, j - i));
    i = j - 1;
  }
  return out;
}

bool Inst::is_terminator() const {
  return opcode == "br" || opcode == "ret" || opcode == "switch" || opcode == "unreachable" ||
         opcode == "indirectbr" || opcode == "resume";
}

Inst parse_inst(const std::string &line) {
  Inst in;
  in.text = line;
  std::string t = trim(strip_comment(line));
  std::string body = t;
  if (starts_with(t, "%")) {
    size_t eq = t.find(" = ");
    if (eq != std::string::npos) {
      in.result = t.substr(0, eq);
      body = trim(t.substr(eq + 3));
    }
  }
  std::vector<std::string> w = words(body);
  size_t k = 0;
  while (k < w.size() && (w[k] == "tail" || w[k] == "musttail" || w[k] == "notail")) ++k;
  if (k < w.size()) in.opcode = w[k];
  std::string after = body.substr(std::min(body.size(), body.find(in.opcode) + in.opcode.size()));
  // skip flags
  auto skip_flags = [&](std::string s) {
    s = trim(s);
    for (;;) {
      std::string first = s.substr(0, s.find(' '));
      if (kFlags.count(first)) {
        s = trim(s.substr(first.size()));
      } else {
        break;
      }
    }
    return s;
  };
  if (!in.result.empty()) {
    const std::string &op = in.opcode;
    if (op == "load") {
      in.type = leading_type(skip_flags(after));
    } else if (op == "phi" || kBinops.count(op) || op == "alloca" || op == "freeze") {
      in.type = op == "alloca" ? "ptr" : leading_type(skip_flags(after));
    } else if (op == "icmp" || op == "fcmp") {
      in.type = "i1";
    } else if (op == "select") {
      std::string s = skip_flags(after);
      size_t c = s.find(',');
      in.type = c == std::string::npos ? "" : leading_type(s.substr(c + 1));
    } else if (kCasts.count(op)) {
      size_t to = after.rfind(" to ");
      in.type = to == std::string::npos ? "" : leading_type(after.substr(to + 4));
    } else if (op == "getelementptr") {
      std::string s = skip_flags(after);
      size_t c = s.find(',');
      in.type = c == std::string::npos ? "ptr" : leading_type(s.substr(c + 1));
    } else if (op == "call") {
      std::string s = skip_flags(after);
      // skip calling-convention / return attributes that are plain words
      std::vector<std::string> cw = words(s);
      size_t i = 0;
      while (i < cw.size() && (cw[i] == "noundef" || cw[i] == "fastcc" || cw[i] == "ccc" ||
                               cw[i] == "zeroext" || cw[i] == "signext" || kFlags.count(cw[i])))
        ++i;
      std::string rest;
      for (size_t j = i; j < cw.size(); ++j) rest += (j > i ? " " : "") + cw[j];
      in.type = leading_type(rest);
    } else if (op == "atomicrmw") {
      std::string s = skip_flags(after);
      std::vector<std::string> cw = words(s);  // op ptr %p, ty %v ...
      size_t c = s.find(',');
      in.type = c == std::string::npos ? "" : leading_type(s.substr(c + 1));
    } else if (op == "extractelement" || op == "extractvalue") {
      in.type = "";
    }
  }
  for (const std::string &v : value_tokens(strip_comment(line)))
    if (v != in.result) in.operands.push_back(v);
  return in;
}

bool uses(const Inst &inst, const std::string &value) {
  for (const std::string &o : inst.operands)
    if (o == value) return true;
  return false;
}

void replace_uses(Inst &inst, const std::string &from, const std::string &to) {
  if (!uses(inst, from)) return;
  std::string &s = inst.text;
  std::string out;
  bool in_str = false;
  // do not rename the result definition itself
  size_t start = 0;
  if (!inst.result.empty()) {
    size_t eq = s.find(inst.result + " = ");
    if (eq != std::string::npos) {
      out = s.substr(0, eq + inst.result.size());
      start = eq + inst.result.size();
    }
  }
  for (size_t i = start; i < s.size(); ++i) {
    if (s[i] == '"') in_str = !in_str;
    if (!in_str && s.compare(i, from.size(), from) == 0 && (i == 0 || !name_char(s[i - 1])) &&
        (i + from.size() == s.size() || !name_char(s[i + from.size()]))) {
      out += to;
      i += from.size() - 1;
      continue;
    }
    out += s[i];
  }
  s = out;
  for (std::string &o : inst.operands)
    if (o == from) o = to;
}

std::string Function::unique(const std::string &base) {
  std::string n = base;
  for (int i = 1; names.count(n); ++i) n = base + "." + std::to_string(i);
  names.insert(n);
  return n;
}

Block *Function::block(const std::string &label) {
  for (Block &b : blocks)
    if (b.label == label) return &b;
  return nullptr;
}

int Function::block_index(const std::string &label) const {
  for (size_t i = 0; i < blocks.size(); ++i)
    if (blocks[i].label == label) return (int)i;
  return -1;
}

static void parse_params(Function &f) {
  const std::string &h = f.header;
  size_t at = h.find("@" + f.name);
  size_t open = h.find('(', at);
  if (open == std::string::npos) return;
  int depth = 0;
  size_t close = open;
  for (size_t i = open; i < h.size(); ++i) {
    if (h[i] == '(') ++depth;
    if (h[i] == ')' && --depth == 0) {
      close = i;
      break;
    }
  }
  std::string inner = h.substr(open + 1, close - open - 1);
  std::vector<std::string> parts;
  depth = 0;
  std::string cur;
  for (char c : inner) {
    if (c == '(' || c == '<' || c == '[' || c == '{') ++depth;
    if (c == ')' || c == '>' || c == ']' || c == '}') --depth;
    if (c == ',' && depth == 0) {
      parts.push_back(trim(cur));
      cur.clear();
    } else {
      cur += c;
    }
  }
  if (!trim(cur).empty()) parts.push_back(trim(cur));
  for (const std::string &p : parts) {
    f.param_types.push_back(leading_type(p));
    std::vector<std::string> v = value_tokens(p);
    f.param_names.push_back(v.empty() ? "" : v.back());
    if (!v.empty()) f.names.insert(v.back());
  }
}

Module parse(const std::string &text) {
  Module m;
  std::istringstream is(text);
  std::string line;
  std::vector<std::string> all;
  while (std::getline(is, line)) all.push_back(line);
  for (size_t i = 0; i < all.size(); ++i) {
    const std::string &l = all[i];
    if (starts_with(l, "define ")) {
      Function f;
      f.header = l;
      size_t at = l.find('@');
      size_t e = at + 1;
      while (e < l.size() && name_char(l[e])) ++e;
      f.name = l.substr(at + 1, e - at - 1);
      f.is_kernel = l.find("ptx_kernel") != std::string::npos;
      parse_params(f);
      Block cur;
      bool have = false;
      for (++i; i < all.size() && trim(all[i]) != "}"; ++i) {
        const std::string &b = all[i];
        std::string tb = trim(strip_comment(b));
        if (tb.empty()) continue;
        bool is_label = !std::isspace(static_cast<unsigned char>(b[0])) && tb.back() == ':';
        if (is_label) {
          if (have || !cur.insts.empty()) f.blocks.push_back(cur);
          cur = Block();
          cur.label = tb.substr(0, tb.size() - 1);
          cur.label_line = b;
          have = true;
          continue;
        }
        Inst in = parse_inst(b);
        if (!in.result.empty()) f.names.insert(in.result);
        cur.insts.push_back(in);
      }
      f.blocks.push_back(cur);
      m.lines.push_back(kFuncMark + std::to_string(m.functions.size()));
      m.functions.push_back(f);
      continue;
    }
    if (l.find("\"target-cpu\"=\"") != std::string::npos) {
      size_t p = l.find("\"target-cpu\"=\"") + 14;
      m.target_cpu = l.substr(p, l.find('"', p) - p);
    }
    if (l.find("!\"kernel\"") != std::string::npos) {
      size_t at = l.find('@');
      if (at != std::string::npos) {
        size_t e = at + 1;
        while (e < l.size() && name_char(l[e])) ++e;
        m.kernel_names.insert(l.substr(at + 1, e - at - 1));
      }
    }
    m.lines.push_back(l);
  }
  for (Function &f : m.functions)
    if (m.kernel_names.count(f.name)) f.is_kernel = true;
  return m;
}

bool Module::has_global(const std::string &name) const {
  for (const std::string &l : lines)
    if (starts_with(l, name + " ") || starts_with(l, name + "=")) return true;
  return false;
}

bool Module::has_declaration(const std::string &name) const {
  for (const std::string &l : lines)
    if (starts_with(l, "declare ") && l.find(name + "(") != std::string::npos) return true;
  for (const Function &f : functions)
    if ("@" + f.name == name) return true;
  return false;
}

void Module::add_global(const std::string &line) {
  for (size_t i = 0; i < lines.size(); ++i)
    if (starts_with(lines[i], kFuncMark) || starts_with(lines[i], "declare ")) {
      lines.insert(lines.begin() + i, line);
      return;
    }
  lines.push_back(line);
}

void Module::add_declaration(const std::string &line) {
  if (!has_declaration(line.substr(line.find('@'), line.find('(') - line.find('@'))))
    lines.push_back(line);
}

std::string Module::print() const {
  std::ostringstream os;
  for (const std::string &l : lines) {
    if (starts_with(l, kFuncMark)) {
      const Function &f = functions[std::stoi(l.substr(std::string(kFuncMark).size()))];
      os << f.header << "\n";
      for (size_t bi = 0; bi < f.blocks.size(); ++bi) {
        const Block &b = f.blocks[bi];
        if (!b.label.empty()) {
          os << (b.label_line.empty() ? b.label + ":" : b.label_line) << "\n";
        }
        for (const Inst &in : b.insts) os << in.text << "\n";
      }
      os << "}\n";
    } else {
      os << l << "\n";
    }
  }
  return os.str();
}

}  // namespace weave
