"""torchrun worker: the sequence-parallel path (GEMM -> reduce-scatter,
owner's reduce + residual + RMSNorm + all-gather, ready-gated GEMM) against
the fused all-reduce path on the same inputs, and TP engine generation in
mode "sp" against mode "fused"."""
import faulthandler
import json
import math
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

from sched_pass_b200 import ops  # noqa: E402
from sched_pass_b200.parallel.tp import TensorParallel, init_distributed  # noqa: E402


def bits(t):
    return t.contiguous().cpu().view(torch.int16).numpy()


faulthandler.enable()  # a native crash prints the Python stack of every thread


def main():
    rank, world, local = init_distributed("nccl", timeout_s=60)
    dev = torch.device("cuda", local)
    out = {"rank": rank, "checks": []}
    fused = TensorParallel(mode="fused", device=dev)
    sptp = TensorParallel(mode="sp", device=dev)
    H, eps = 1024, 1e-5
    sp = sptp.sequence_parallel(H, 512)
    g = torch.Generator(device="cpu").manual_seed(99)
    lnw = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(dev)
    w2 = (torch.randn(768, H, generator=g) / math.sqrt(H)).to(torch.bfloat16).to(dev)
    # token counts shrink and grow (stale flags), and include T < world
    for call, (T, K) in enumerate([(16, 512), (100, 256), (1, 512), (5, 1024), (300, 256), (16, 512)]):
        x_full = torch.randn(T, K * world, generator=g)
        w_full = torch.randn(H, K * world, generator=g) / math.sqrt(K * world)
        x = x_full[:, rank * K:(rank + 1) * K].to(torch.bfloat16).to(dev).contiguous()
        w = w_full[:, rank * K:(rank + 1) * K].to(torch.bfloat16).to(dev).contiguous()
        res0 = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
        # fused all-reduce + add_rmsnorm
        y = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        fused.linear_allreduce(x, w, y)
        res_a = res0.clone()
        normed_a = ops.add_rmsnorm(y, res_a, lnw, eps)
        # sequence parallel
        res_b = res0.clone()
        delta = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)
        sp.linear_rs(x, w)
        normed_b, ready = sp.reduce_norm(res_b, lnw, eps, T, delta=delta)
        z_gated = ops.linear(normed_b, w2, x_ready=ready)  # waits per token tile
        sp.wait_rows(ready, T)
        z_plain = ops.linear(normed_b.clone(), w2)
        torch.cuda.synchronize()
        lo, hi = sp.owned(T)
        c = {"T": T, "K": K, "rows": [lo, hi],
             "delta_bits": bool(np.array_equal(bits(delta[lo:hi]), bits(y[lo:hi]))),
             "residual_bits": bool(np.array_equal(bits(res_b[lo:hi]), bits(res_a[lo:hi]))),
             "normed_bits": bool(np.array_equal(bits(normed_b), bits(normed_a))),
             "gated_gemm_bits": bool(np.array_equal(bits(z_gated), bits(z_plain)))}
        ns = [torch.empty_like(normed_b) for _ in range(world)]
        dist.all_gather(ns, normed_b.contiguous())
        c["identical_on_ranks"] = all(torch.equal(ns[0], n) for n in ns)
        out["checks"].append(c)
    ops.check_status()
    # engine: mode "sp" == mode "fused" (the same arithmetic, so the same tokens)
    from sched_pass_b200.engine.engine import Engine, EngineConfig
    from sched_pass_b200.models.config import LLAMA_TINY, ModelConfig
    from sched_pass_b200.models.llama import full_weights, shard_weights
    cfg = LLAMA_TINY if LLAMA_TINY.n_kv_heads % world == 0 else ModelConfig(
        "llama-tiny-kv8", 2, 512, 8, 8, 128, 1024, 1024)
    full = full_weights(cfg, seed=5)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, cfg.vocab, size=int(n)).astype(np.int32) for n in (9, 70, 33, 3)]
    ecfg = dict(max_batch=8, max_prefill_tokens=256, max_context=512)
    res = {}
    for mode, tp in (("fused", fused), ("sp", sptp)):
        eng = Engine(cfg, EngineConfig(**ecfg), dev, tp=tp, weights=shard_weights(cfg, full, rank, world, dev))
        res[mode] = eng.generate(prompts, max_new_tokens=6)
        eng.graphs.clear()
        del eng
        torch.cuda.synchronize()
    ops.check_status()
    out["tokens_fused"] = res["fused"]
    out["tokens_sp"] = res["sp"]
    out["engine_identical"] = res["fused"] == res["sp"]
    out["sp_calls"] = [sp.calls_rs, sp.calls_ag]
    dist.barrier()
    if rank == 0:
        print("SPJSON " + json.dumps(out))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
