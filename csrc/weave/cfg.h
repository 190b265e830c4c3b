// cfg.h -- control-flow analysis over the weaver's IR model.
//
// The reference weaver asks LLVM for LoopInfo, DominatorTree and
// ScalarEvolution (jc-su/sched-pass lib/SchedWeave.cpp:1054-1088, the
// canonical-IV shed at :652-704). Without LLVM libraries the same facts are
// computed here from the blocks' terminators:
//   * successors / predecessors (every `label %x` of a block's terminator,
//     including the case lines of a multi-line `switch`);
//   * the dominator tree, by the iterative algorithm of Cooper, Harvey and
//     Kennedy ("A Simple, Fast Dominance Algorithm", 2001) over reverse
//     postorder;
//   * natural loops: an edge t -> h is a back edge when h dominates t; the
//     loop of header h is h plus every block that reaches a back-edge tail
//     without passing through h (all back edges to one header form one loop);
//   * the canonical induction variable of a loop, structurally: an integer
//     phi of the header whose incoming value is the constant 0 on every edge
//     from outside the loop and, on every back edge, a value defined as
//     `add <ty> %iv, 1` (either operand order, any wrap flags).
// Block indices are positions in Function::blocks; the passes only append
// blocks, so indices computed before an edit stay valid.
#pragma once

#include <functional>
#include <string>
#include <vector>

#include "ir.h"

namespace weave {

struct Cfg {
  std::vector<std::vector<int>> succ, pred;
  std::vector<int> rpo;        // reachable blocks, reverse postorder from the entry
  std::vector<int> rpo_index;  // position of a block in rpo; -1 if unreachable
  std::vector<int> idom;       // immediate dominator; the entry's is itself, -1 if unreachable

  explicit Cfg(const Function &f);
  bool reachable(int b) const { return b >= 0 && b < (int)rpo_index.size() && rpo_index[b] >= 0; }
  // a dominates b (reflexive); false if either is unreachable
  bool dominates(int a, int b) const;
};

struct NaturalLoop {
  int header = -1;
  std::vector<int> latches;  // tails of the back edges into the header
  std::vector<char> body;    // body[b] != 0 for every block of the loop
  int size = 0;              // blocks in the body
  std::string iv;            // canonical induction variable ("%name"), "" if none
  std::string iv_type;
  bool contains(int b) const { return b >= 0 && b < (int)body.size() && body[b]; }
};

// Labels named by `label %x` in the text of a terminator line.
std::vector<std::string> branch_labels(const std::string &text);

// Incoming pairs of a phi line: (value text, block label without '%').
std::vector<std::pair<std::string, std::string>> phi_incoming(const std::string &phi_text);

// Natural loops of f, outermost first for each header order (sorted by header
// position in reverse postorder); each with its canonical IV if it has one.
std::vector<NaturalLoop> natural_loops(const Function &f, const Cfg &g);

// The loop-carried canonical IV of loop L, or "" (fills L.iv / L.iv_type).
void find_canonical_iv(const Function &f, NaturalLoop &L);

// Rewrite the incoming values of a phi: `from` becomes `to` on the edges
// whose predecessor label satisfies keep(label). Returns true if changed.
bool rewrite_phi_incoming(Inst &phi, const std::string &from, const std::string &to,
                          const std::function<bool(const std::string &)> &keep);

}  // namespace weave
