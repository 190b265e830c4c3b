"""Run the C++ IR weaver (csrc/weave) on LLVM assembly text.

``weave(text, env)`` is the equivalent of
``opt -load-pass-plugin=... -passes=sched-workqueue,sched-weave``: the
environment carries the SCHED_* knobs exactly as for the reference plugin.
"""
from __future__ import annotations

import os
import subprocess

from .. import _build


def weaver_path() -> str:
    path = _build.build_weaver()
    if path is None:
        raise RuntimeError("the weaver sources are missing")
    return path


def weave(text: str, env: dict | None = None, passes: str = "sched-workqueue,sched-weave",
          debug: bool = True) -> tuple[str, list[str]]:
    """Returns (woven text, notes). ``env`` entries override os.environ;
    a value of None removes the variable."""
    e = dict(os.environ)
    for k in list(e):
        if k.startswith("SCHED_") and k not in (env or {}):
            e.pop(k)  # only the explicit knobs reach the weave
    for k, v in (env or {}).items():
        if v is None:
            e.pop(k, None)
        else:
            e[k] = str(v)
    if debug:
        e["SCHED_DEBUG"] = "1"
    r = subprocess.run([weaver_path(), f"--passes={passes}", "-"], input=text, capture_output=True,
                       text=True, env=e, check=False)
    if r.returncode != 0:
        raise RuntimeError(f"sched-weave failed ({r.returncode}): {r.stderr[-2000:]}")
    notes = [l[len("[sched] "):] for l in r.stderr.splitlines() if l.startswith("[sched] ")]
    return r.stdout, notes


def manifest_csv() -> list[dict]:
    r = subprocess.run([weaver_path(), "--manifest=csv"], capture_output=True, text=True, check=True)
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    hdr = lines[0].split(",")
    return [dict(zip(hdr, l.split(","))) for l in lines[1:]]
