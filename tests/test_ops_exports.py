"""Every ``ops.<name>`` the models, engine and parallel layers call is
exported by the package (a missing export only shows up on a GPU box
otherwise, where the forward runs)."""
import os
import re

import sched_pass_b200.ops as ops

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_ops_names_used_by_the_package_exist():
    used = set()
    pkg = os.path.join(ROOT, "sched_pass_b200")
    for d, _, files in os.walk(pkg):
        for f in files:
            if f.endswith(".py"):
                text = open(os.path.join(d, f)).read()
                used |= set(re.findall(r"\bops\.([a-z_]\w*)\(", text))
    missing = sorted(n for n in used if not hasattr(ops, n))
    assert not missing, missing
