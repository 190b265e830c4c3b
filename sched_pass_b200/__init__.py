"""sched_pass_b200 -- a Blackwell-native (sm_100a) late-bound scheduling
runtime for continuous-batching LLM decode.

Subpackages:
  runtime   control tables (ABI-compatible SchedPlane/SchedArena), manifest,
            closed-loop controller
  compiler  the LLVM-IR weaver driver and NVPTX code generation
  ops       tensor entry points of the sm_100a kernels
  models    Llama / Mixtral architectures, pure-PyTorch oracles
  parallel  symmetric peer memory, fused GEMM+collective TP, expert parallel
  engine    continuous-batching engine, paged KV, tiered KV, workloads
  utils     device timing, clock sampling
"""
__version__ = "0.1.0"
