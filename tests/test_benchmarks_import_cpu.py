"""Every benchmark module imports on a CPU host and exposes ``main`` (the
GPU work happens only when ``main`` runs), so a broken benchmark shows up
here rather than on the GPU box."""
import importlib
import pkgutil

import pytest

import sched_pass_b200.benchmarks as bm

LIBRARIES = ("common", "steady_state")  # helpers the benchmarks and bench.py import
MODULES = sorted(m.name for m in pkgutil.iter_modules(bm.__path__) if m.name not in LIBRARIES)


@pytest.mark.parametrize("name", MODULES)
def test_benchmark_module_imports(name):
    mod = importlib.import_module(f"sched_pass_b200.benchmarks.{name}")
    assert callable(getattr(mod, "main", None)), f"{name} has no main()"


@pytest.mark.parametrize("name", LIBRARIES)
def test_benchmark_library_imports(name):
    importlib.import_module(f"sched_pass_b200.benchmarks.{name}")
