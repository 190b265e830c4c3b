// main.cpp -- the `sched-weave` command line (the pass pipeline driver).
//
//   sched-weave [--passes=sched-workqueue,sched-weave] [-o out.ll] [in.ll|-]
//   sched-weave --manifest[=csv]
//
// Plays the role of `opt -load-pass-plugin=... -passes=sched-weave`: reads
// LLVM assembly, runs the work-queue transform (only when SCHED_WORKQUEUE is
// set) and then the weave, in the manifest's order, and prints the result.
// Configuration comes from the same SCHED_* environment knobs. With
// SCHED_DEBUG the passes' notes (what was woven, what was declined and why)
// go to stderr. SCHED_MANIFEST_DUMP[=csv] also prints the manifest.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <sstream>

#include "passes.h"
#include "sched/manifest.h"

using namespace weave;

static void dump_manifest(bool csv) {
  for (unsigned i = 1; i < sched::kNumLevers; ++i)
    if (sched::kLevers[i].order < sched::kLevers[i - 1].order)
      std::cerr << "[sched] manifest order broken at " << sched::kLevers[i].name << "\n";
  if (csv) {
    std::cout << "name,effect,minSm,knob,disableKnob,order,tag\n";
    for (const sched::Lever &l : sched::kLevers)
      std::cout << l.name << ',' << sched::effect_name(l.effect) << ',' << l.min_sm << ',' << l.knob << ','
                << (l.knob_disables ? 1 : 0) << ',' << l.order << ',' << l.tag << '\n';
    return;
  }
  std::cout << "== sched lever manifest (" << sched::kNumLevers << " levers) ==\n";
  for (const sched::Lever &l : sched::kLevers) {
    std::cout << "  [" << l.order << "] " << l.name << "  " << sched::effect_name(l.effect) << "  sm>=" << l.min_sm
              << "  knob=" << l.knob << (l.knob_disables ? " (disables)" : " (enables)") << "  slots=" << l.slots;
    if (l.tag[0]) std::cout << "  tag=" << l.tag;
    std::cout << "\n      " << l.contract << "\n";
  }
}

int main(int argc, char **argv) {
  std::string passes = "sched-workqueue,sched-weave", in = "-", out = "-";
  bool manifest = false, csv = false;
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i];
    if (a.rfind("--passes=", 0) == 0 || a.rfind("-passes=", 0) == 0) {
      passes = a.substr(a.find('=') + 1);
    } else if (a == "--manifest" || a == "--manifest=text") {
      manifest = true;
    } else if (a == "--manifest=csv") {
      manifest = csv = true;
    } else if (a == "-o" && i + 1 < argc) {
      out = argv[++i];
    } else if (a == "-S") {
      // accepted for opt compatibility (output is always text)
    } else if (a == "-h" || a == "--help") {
      std::cout << "usage: sched-weave [--passes=sched-workqueue,sched-weave] [-o out.ll] [in.ll|-]\n"
                   "       sched-weave --manifest[=csv]\n";
      return 0;
    } else {
      in = a;
    }
  }
  if (const char *d = std::getenv("SCHED_MANIFEST_DUMP")) {
    dump_manifest(std::strcmp(d, "csv") == 0);
    if (manifest) return 0;
  }
  if (manifest) {
    dump_manifest(csv);
    return 0;
  }
  std::stringstream buf;
  if (in == "-") {
    buf << std::cin.rdbuf();
  } else {
    std::ifstream f(in);
    if (!f) {
      std::cerr << "sched-weave: cannot read " << in << "\n";
      return 2;
    }
    buf << f.rdbuf();
  }
  Module m = parse(buf.str());
  Config c = Config::from_env();
  Notes notes;
  // manifest order: the work queue runs before the weave
  if (passes.find("sched-workqueue") != std::string::npos) run_workqueue(m, c, notes);
  if (passes.find("sched-weave") != std::string::npos) run_weave(m, c, notes);
  if (c.debug)
    for (const std::string &n : notes.lines) std::cerr << "[sched] " << n << "\n";
  std::string text = m.print();
  if (out == "-") {
    std::cout << text;
  } else {
    std::ofstream f(out);
    f << text;
  }
  return 0;
}
