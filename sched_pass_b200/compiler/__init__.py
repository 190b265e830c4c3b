"""Compiler plane: the IR weaver (``sched-weave``, C++), CPU execution of
woven IR for host-only checks, and NVPTX code generation + loading for GPU
fixtures of IR-woven kernels."""
