// sched/manifest.h -- the lever registry: one row per woven capability.
//
// Every consumer derives from this table instead of keeping its own list:
//   * the IR weaver (csrc/weave) applies levers in row order and reads each
//     row's knob to decide whether it is compiled in;
//   * the source-level weave points (weave.cuh) expose one template flag per
//     row, and the kernel-variant cache key is built from the rows' tags;
//   * `sched-weave --manifest[=csv]` prints it, and the Python mirror
//     (sched_pass_b200/runtime/manifest.py) is checked against that dump.
//
// The six rows, their effect classes and ordering constraints are the ones
// of the reference's include/sched/SchedManifest.h:76-105 (kept identical so
// the two control planes agree on knob names and cache tags):
//   workqueue before every other lever (it creates the task-body the others
//   instrument); shed before policy (policy splits blocks); the claim after
//   the body; pi honoured only when order_size equals the launch size.
#pragma once

namespace sched {

enum class Effect : int {
  Hint = 0,     // E0: cannot change results (prefetch, discard, PDL)
  Permute = 1,  // E1: reorders disjoint tasks (pi) -- bit-exact
  Budget = 2,   // E2: bounded-accuracy truncation (shed, tau > 0 only)
  Observe = 3,  // O : commutative accumulation (timer) -- replay-safe
  Acquire = 4,  // launch-model change (ticket / cluster launch control)
};

constexpr const char *effect_name(Effect e) {
  return e == Effect::Hint      ? "E0/hint"
         : e == Effect::Permute ? "E1/permute"
         : e == Effect::Budget  ? "E2/budget"
         : e == Effect::Observe ? "O/observe"
                                : "acquire";
}

struct Lever {
  const char *name;
  Effect effect;
  unsigned min_sm;     // lowest sm_NN that supports it (0 = any)
  const char *slots;   // runtime slots it reads
  const char *knob;    // environment knob controlling it at weave time
  bool knob_disables;  // true: SCHED_NO_<X> turns it off; false: SCHED_<X> turns it on
  int order;           // weave order, ascending
  const char *tag;     // kernel-cache key fragment ("" = none)
  const char *contract;
};

inline constexpr Lever kLevers[] = {
    {"workqueue", Effect::Acquire, 0, "ctrl(+queue for ticket)", "SCHED_WORKQUEUE", false, 0,
     "-wq",
     "persistent driver; ticket claims need queue+ctrl, cluster-launch-control claims need ctrl; "
     "1-D task grid only; the next claim is issued after the current task finishes"},
    {"pi", Effect::Permute, 0, "order,ctrl", "SCHED_NO_INDIRECT", true, 1, "",
     "task = order[raw]; an entry outside the launch falls back to raw, and the whole launch "
     "uses identity unless ctrl.order_size is 0 or equals the launch size"},
    {"shed", Effect::Budget, 0, "ctrl", "SCHED_NO_SHED", true, 2, "-nos",
     "tau > 0 truncates the task's KV stream to its first tau units (softmax score -> -inf, "
     "linear value -> 0) on the loop's canonical induction variable; tau == 0 is bit-exact"},
    {"policy", Effect::Hint, 80, "ctrl", "SCHED_NO_POLICY", true, 3, "-nop",
     "urgent (hint 1, or hint 0 with q*dT - lambda_bw*dR - H > 0): L2 evict_last prefetch "
     "ahead of the stream; polite (hint 2): demote consumed lines to normal L2 priority"},
    {"timer", Effect::Observe, 0, "timer,ctrl", "SCHED_NO_TIMER", true, 4, "-ti",
     "clock64 bracket, thread 0 adds the task's cycles to timer[task]; ctrl.flags bit0 is read "
     "once at entry and switches this launch's write off"},
    {"pdl", Effect::Hint, 90, "-", "SCHED_PDL", false, 5, "",
     "griddepcontrol.wait after the table reads, launch_dependents before exit; no-op unless "
     "the launch enables programmatic stream serialization"},
};

inline constexpr unsigned kNumLevers = sizeof(kLevers) / sizeof(kLevers[0]);

inline const Lever *lever_by_name(const char *name) {
  for (const Lever &l : kLevers) {
    const char *a = l.name, *b = name;
    while (*a && *a == *b) ++a, ++b;
    if (!*a && !*b) return &l;
  }
  return nullptr;
}

}  // namespace sched
