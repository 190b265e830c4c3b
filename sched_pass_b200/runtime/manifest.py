"""Python mirror of the lever registry (include/sched/manifest.h).

Row order is the weave order. ``tests/test_weave_ir.py`` checks this mirror
against the C++ table, dumped by ``sched-weave --manifest=csv``.
Fields: name, effect, min_sm, knob, knob_disables, tag.

``python -m sched_pass_b200.runtime.manifest`` prints the table as markdown
(the reference generates the same document from its C++ manifest,
scripts/gen_manifest_doc.sh).
"""
from __future__ import annotations

MANIFEST = [
    ("workqueue", "acquire", 0, "SCHED_WORKQUEUE", False, "-wq"),
    ("pi", "E1/permute", 0, "SCHED_NO_INDIRECT", True, ""),
    ("shed", "E2/budget", 0, "SCHED_NO_SHED", True, "-nos"),
    ("policy", "E0/hint", 80, "SCHED_NO_POLICY", True, "-nop"),
    ("timer", "O/observe", 0, "SCHED_NO_TIMER", True, "-ti"),
    ("pdl", "E0/hint", 90, "SCHED_PDL", False, ""),
]

LEVER_NAMES = [row[0] for row in MANIFEST]


def disable_mask(env) -> str:
    """Cache-key fragment of the lever-disable knobs present in ``env``:
    one letter per SCHED_NO_<WORD> knob (its first letter), in manifest order."""
    return "".join(knob[len("SCHED_NO_"):][0].lower()
                   for _n, _e, _sm, knob, disables, _t in MANIFEST
                   if disables and env.get(knob))


def levers_enabled(env) -> dict:
    """Which levers a weave under ``env`` compiles in."""
    out = {}
    for name, _e, _sm, knob, disables, _t in MANIFEST:
        present = bool(env.get(knob))
        out[name] = (not present) if disables else present
    return out


def manifest_markdown() -> str:
    """The lever table as markdown, one row per lever in weave order."""
    lines = ["| order | lever | effect | min SM | knob | knob disables | cache tag |",
             "|---|---|---|---|---|---|---|"]
    for i, (name, effect, min_sm, knob, disables, tag) in enumerate(MANIFEST):
        lines.append(f"| {i} | {name} | {effect} | {min_sm or '-'} | `{knob}` | {'yes' if disables else 'no (enables)'} "
                     f"| {('`' + tag + '`') if tag else '-'} |")
    return "\n".join(lines)


if __name__ == "__main__":
    print(manifest_markdown())
