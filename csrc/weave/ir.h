// ir.h -- a small textual model of LLVM IR modules for the weaver.
//
// The weaver edits LLVM assembly text directly (no LLVM libraries are
// linked): a module is kept as its top-level lines plus parsed function
// bodies; a function is a list of basic blocks; an instruction is its text
// with the few parsed facts the passes need (result name, opcode, result
// type, operand value names). Edits insert or rewrite instruction text and
// rename value uses; everything not touched is printed back verbatim, so the
// output stays the input plus the woven code. Values the weaver creates are
// always named (`%sched.*`), so the numbering of unnamed values is never
// disturbed.
#pragma once

#include <map>
#include <set>
#include <string>
#include <vector>

namespace weave {

struct Inst {
  std::string text;    // full line without trailing newline
  std::string result;  // "%name" or ""
  std::string opcode;  // "load", "call", "br", "phi", ...
  std::string type;    // result type ("i32", "float", "ptr", "i1", ...), "" if none
  std::vector<std::string> operands;  // value names used (in textual order, "%x")
  bool is_terminator() const;
};

struct Block {
  std::string label;       // without '%' / ':' ; "" for an unlabelled entry block
  std::string label_line;  // original label line ("" if none)
  std::vector<Inst> insts;
};

struct Function {
  std::string name;        // without '@'
  std::string header;      // "define ... {"
  std::vector<Block> blocks;
  bool is_kernel = false;
  std::vector<std::string> param_types;
  std::vector<std::string> param_names;
  int fresh = 0;

  std::string unique(const std::string &base);  // "%sched.x", "%sched.x.1", ...
  std::set<std::string> names;                  // defined value names
  Block *block(const std::string &label);
  int block_index(const std::string &label) const;
};

// Placeholder line standing for function i in Module::lines.
constexpr const char *kFuncMark = "\x01" "FUNC:";

struct Module {
  std::vector<std::string> lines;   // top-level text; functions are placeholders
  std::vector<Function> functions;  // in order; placeholder kFuncMark + i in lines
  std::string target_cpu;           // "sm_100a" etc. from attributes, if present
  std::set<std::string> kernel_names;  // from !nvvm.annotations

  bool has_global(const std::string &name) const;  // "@x" defined or declared
  bool has_declaration(const std::string &name) const;
  void add_global(const std::string &line);        // appended before the first function
  void add_declaration(const std::string &line);   // appended at the end
  std::string print() const;
};

Module parse(const std::string &text);
Inst parse_inst(const std::string &line);

// Value uses: replace every token `from` (as a whole value name) by `to` in
// the instruction text, keeping its parsed operand list in sync.
void replace_uses(Inst &inst, const std::string &from, const std::string &to);
bool uses(const Inst &inst, const std::string &value);

// Helpers for emitting instruction text.
std::string trim(const std::string &s);
bool starts_with(const std::string &s, const std::string &p);
std::vector<std::string> value_tokens(const std::string &s);

}  // namespace weave
