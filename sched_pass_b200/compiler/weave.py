"""Run the C++ IR weaver (csrc/weave) on LLVM assembly text.

``weave(text, env)`` is the equivalent of
``opt -load-pass-plugin=... -passes=sched-workqueue,sched-weave``: the
environment carries the SCHED_* knobs exactly as for the reference plugin.

``weave_cached(text, env, name)`` keeps the woven module in the directory
``env["SCHED_KERNEL_CACHE"]`` (chosen by ``runtime.sched_rt.compute_bake_env``
from the arena's VA, capacity, lever mask and weaver hash), under a name
that also hashes the source and every SCHED_* knob. A later process whose
arena lands on the same VA finds the same entry and reuses it, as the
reference reuses its JIT ``.so`` across processes (test/py/test_fixed_va.py).
"""
from __future__ import annotations

import hashlib
import json
import os
import subprocess
import tempfile

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


def weave_cached(text: str, env: dict, name: str = "kernel",
                 passes: str = "sched-workqueue,sched-weave") -> tuple[str, list[str], bool]:
    """``weave`` through a content-addressed cache in
    ``env["SCHED_KERNEL_CACHE"]``. Returns (woven text, notes, cache hit).
    Entries are written atomically (temporary file + rename), so concurrent
    processes never read a partial one."""
    root = env.get("SCHED_KERNEL_CACHE")
    if not root:
        raise ValueError("env has no SCHED_KERNEL_CACHE (see compute_bake_env)")
    knobs = {k: str(v) for k, v in sorted(env.items()) if k.startswith("SCHED_") and k != "SCHED_KERNEL_CACHE"}
    h = hashlib.sha256()
    h.update(text.encode())
    h.update(json.dumps([passes, knobs]).encode())
    h.update(_file_hash(weaver_path()).encode())
    path = os.path.join(root, f"{name}-{h.hexdigest()[:16]}.ll")
    notes_path = path + ".notes"
    if os.path.exists(path) and os.path.exists(notes_path):
        with open(path) as f, open(notes_path) as g:
            return f.read(), g.read().splitlines(), True
    out, notes = weave(text, env, passes)
    os.makedirs(root, exist_ok=True)
    for dst, body in ((notes_path, "\n".join(notes)), (path, out)):  # the module last: it marks the entry
        fd, tmp = tempfile.mkstemp(dir=root, prefix=".tmp-")
        with os.fdopen(fd, "w") as f:
            f.write(body)
        os.replace(tmp, dst)
    return out, notes, False


def _file_hash(path: str) -> str:
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()[:16]


def manifest_csv() -> list[dict]:
    r = subprocess.run([weaver_path(), "--manifest=csv"], capture_output=True, text=True, check=True)
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    hdr = lines[0].split(",")
    return [dict(zip(hdr, l.split(","))) for l in lines[1:]]
