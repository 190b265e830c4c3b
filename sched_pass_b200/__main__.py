"""Command line of the framework:

    python -m sched_pass_b200 build                      compile the native parts (sm_100a)
    python -m sched_pass_b200 weave IN.ll [-o OUT.ll] [--env K=V ...]
                                                          weave the levers into LLVM IR
    python -m sched_pass_b200 manifest [--csv]           the lever table
    python -m sched_pass_b200 serve [server options]     HTTP server (engine/server.py)
    python -m sched_pass_b200 loadgen [loadgen options]  load generator (engine/loadgen.py)
    python -m sched_pass_b200 doctor                     what this machine offers the framework
"""
from __future__ import annotations

import argparse
import sys


def _weave(argv) -> int:
    from .compiler.weave import weave
    ap = argparse.ArgumentParser(prog="sched_pass_b200 weave")
    ap.add_argument("src")
    ap.add_argument("-o", "--out", default="-")
    ap.add_argument("--env", action="append", default=[], help="SCHED_* knob as KEY=VALUE (repeatable)")
    ap.add_argument("--passes", default="sched-workqueue,sched-weave")
    a = ap.parse_args(argv)
    env = {}
    for kv in a.env:
        k, _, v = kv.partition("=")
        if not k.startswith("SCHED_"):
            ap.error(f"--env expects SCHED_* knobs, not {k!r}")
        env[k] = v
    with open(a.src) as f:
        text = f.read()
    out, notes = weave(text, env, a.passes)
    for n in notes:
        print("[sched] " + n, file=sys.stderr)
    if a.out == "-":
        sys.stdout.write(out)
    else:
        with open(a.out, "w") as f:
            f.write(out)
    return 0


def _manifest(argv) -> int:
    ap = argparse.ArgumentParser(prog="sched_pass_b200 manifest")
    ap.add_argument("--csv", action="store_true", help="the C++ table as sched-weave dumps it")
    a = ap.parse_args(argv)
    if a.csv:
        from .compiler.weave import manifest_csv
        rows = manifest_csv()
        print(",".join(rows[0].keys()))
        for r in rows:
            print(",".join(r.values()))
    else:
        from .runtime.manifest import manifest_markdown
        print(manifest_markdown())
    return 0


def doctor() -> dict:
    """Environment report: toolchain, GPUs (arch, SMs, memory), peer access
    between GPU pairs, NCCL, the native build, and the measured peaks file."""
    import os
    import shutil

    from . import _build
    rep = {"python": sys.version.split()[0]}
    try:
        import torch
        rep["torch"] = torch.__version__
        rep["cuda_runtime"] = torch.version.cuda
        n = torch.cuda.device_count() if torch.cuda.is_available() else 0
        rep["gpus"] = []
        for i in range(n):
            p = torch.cuda.get_device_properties(i)
            rep["gpus"].append({"index": i, "name": p.name, "sm": f"{p.major}{p.minor}",
                                "sms": p.multi_processor_count, "memory_gib": round(p.total_memory / 2 ** 30, 1),
                                "sm_100a_kernels_run": (p.major, p.minor) == (10, 0)})
        rep["peer_access"] = {f"{i}->{j}": torch.cuda.can_device_access_peer(i, j)
                              for i in range(n) for j in range(n) if i != j} if n > 1 else {}
        try:
            rep["nccl"] = ".".join(str(v) for v in torch.cuda.nccl.version())
        except Exception:  # noqa: BLE001 - no NCCL in this torch
            rep["nccl"] = None
    except ImportError:
        rep["torch"] = None
    rep["nvcc"] = shutil.which("nvcc") or ("/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc")
                                           else None)
    rep["native"] = {"extension": os.path.exists(_build.ext_path()),
                     "weaver": os.path.exists(_build.weave_binary()),
                     "host_runtime": os.path.exists(_build.hostlib_path())}
    peaks = os.path.join(os.path.dirname(_build.PKG_DIR), "MEASURED_PEAKS.json")
    rep["measured_peaks"] = peaks if os.path.exists(peaks) else None
    return rep


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] in ("-h", "--help"):
        print(__doc__)
        return 0
    cmd, rest = argv[0], argv[1:]
    if cmd == "build":
        from . import _build
        _build.build_all(verbose="-v" in rest)
        return 0
    if cmd == "weave":
        return _weave(rest)
    if cmd == "manifest":
        return _manifest(rest)
    if cmd == "serve":
        from .engine.server import main as serve_main
        return serve_main(rest)
    if cmd == "doctor":
        import json
        print(json.dumps(doctor(), indent=2))
        return 0
    if cmd == "loadgen":
        from .engine.loadgen import main as loadgen_main
        return loadgen_main(rest)
    print(f"unknown command {cmd!r}\n" + __doc__, file=sys.stderr)
    return 2


if __name__ == "__main__":
    raise SystemExit(main())
