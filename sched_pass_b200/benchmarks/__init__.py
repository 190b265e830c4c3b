"""Runnable microbenchmarks (``python -m sched_pass_b200.benchmarks.<name>``)."""
