"""torchrun worker: fused GEMM + all-reduce vs an fp32 reference, and TP
engine generation vs single-GPU generation on the same logical weights."""
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


faulthandler.enable()  # a native crash prints the Python stack of every thread


def main():
    rank, world, local = init_distributed("nccl", timeout_s=60)
    dev = torch.device("cuda", local)
    out = {"rank": rank, "checks": []}
    tp = TensorParallel(mode="fused", device=dev)
    g = torch.Generator(device="cpu").manual_seed(1234)
    for (T, N, K) in [(1, 4096, 512), (16, 4096, 1024), (100, 1024, 2048), (300, 2048, 512)]:
        x_full = torch.randn(T, K * world, generator=g)
        w_full = torch.randn(N, K * world, generator=g) / math.sqrt(K * world)
        ref = x_full.to(torch.bfloat16).float() @ w_full.to(torch.bfloat16).float().t()
        x = x_full[:, rank * K:(rank + 1) * K].to(torch.bfloat16).to(dev).contiguous()
        w = w_full[:, rank * K:(rank + 1) * K].to(torch.bfloat16).to(dev).contiguous()
        y = torch.empty(T, N, dtype=torch.bfloat16, device=dev)
        for rep in range(3):  # alternating slab sets, flags must reset
            tp.linear_allreduce(x, w, y)
        torch.cuda.synchronize()
        err = ((y.float().cpu() - ref).norm() / ref.norm()).item()
        # the kernel's output is the rank-order reduction of the partials it received (CPU oracle)
        from sched_pass_b200.parallel import protocol
        slab = tp._fused.last_slab(T, N).cpu().view(torch.int16).numpy().view(np.uint16)
        oracle = protocol.reduce_rank_order(slab)
        oracle_ok = bool(np.array_equal(y.cpu().view(torch.int16).numpy().view(np.uint16), oracle))
        ys = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(ys, y)
        same = all(torch.equal(ys[0], z) for z in ys)
        # residual add + RMSNorm inside the fused kernel == the separate kernel
        res0 = torch.randn(T, N, generator=g).to(torch.bfloat16).to(dev)
        nw = (1 + 0.1 * torch.randn(N, generator=g)).to(torch.bfloat16).to(dev)
        r1 = res0.clone()
        n1 = ops.add_rmsnorm(y, r1, nw, 1e-5)
        y2, r2 = torch.empty_like(y), res0.clone()
        n2 = torch.empty_like(r2)
        tp.linear_allreduce(x, w, y2, norm=(r2, nw, 1e-5, n2))
        torch.cuda.synchronize()
        norm_ok = bool(torch.equal(y2, y) and torch.equal(r2, r1) and torch.equal(n2, n1))
        out["checks"].append({"T": T, "N": N, "K": K, "rel_err": err, "identical_on_ranks": same,
                              "matches_protocol_oracle": oracle_ok, "fused_norm_exact": norm_ok})
    ops.check_status()
    print(f"STAGE {rank} fused all-reduce checks done", flush=True)
    # greedy sampling over a vocabulary split across ranks: the in-kernel
    # exchange of (max, id) pairs == the all-gather of the pairs
    H, V = 512, 1000 * world + 7
    vloc = ((V + world - 1) // world + 127) // 128 * 128  # shard rows padded to GEMM row tiles, as the model does
    lm = (torch.randn(vloc * world, H, generator=g) / H ** 0.5).to(torch.bfloat16)
    lm_local = lm[rank * vloc:(rank + 1) * vloc].to(dev).contiguous()
    samples = []
    for S in (1, 6, 100):
        rows = torch.randn(S, H, generator=g).to(torch.bfloat16).to(dev)
        a = torch.empty(S, dtype=torch.int32, device=dev)
        b = torch.empty(S, dtype=torch.int32, device=dev)
        tp.sharded_argmax(rows, lm_local, rank * vloc, V, a)
        saved, tp._sample = tp._sample, None
        tp.sharded_argmax(rows, lm_local, rank * vloc, V, b)
        tp._sample = saved
        torch.cuda.synchronize()
        want = (rows.float().cpu() @ lm[:V].float().t()).argmax(1)
        samples.append({"S": S, "exchange_equals_allgather": bool(torch.equal(a, b)),
                        "agrees_with_fp32": float((a.cpu().long() == want).float().mean())})
    out["sampling"] = samples
    ops.check_status()
    print(f"STAGE {rank} sampling exchange done", flush=True)
    # engine: TP generation == single-GPU generation
    from sched_pass_b200.engine.engine import Engine, EngineConfig
    from sched_pass_b200.models.config import LLAMA_TINY, ModelConfig
    from sched_pass_b200.models.llama import full_weights, shard_weights
    # heads must split evenly over the ranks (LLAMA_TINY has 2 KV heads)
    cfg = LLAMA_TINY if LLAMA_TINY.n_kv_heads % world == 0 else ModelConfig(
        "llama-tiny-kv8", 2, 512, 8, 8, 128, 1024, 1024)
    full = full_weights(cfg, seed=5)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, cfg.vocab, size=int(n)).astype(np.int32) for n in (9, 70, 33)]
    ecfg = dict(max_batch=8, max_prefill_tokens=256, max_context=512)
    eng = Engine(cfg, EngineConfig(**ecfg), dev, tp=tp,
                 weights=shard_weights(cfg, full, rank, world, dev))
    tp_out = eng.generate(prompts, max_new_tokens=5)
    print(f"STAGE {rank} TP engine generated", flush=True)
    del eng
    if rank == 0:
        single = Engine(cfg, EngineConfig(**ecfg), dev,
                        weights=shard_weights(cfg, full, 0, 1, dev))
        ref_out = single.generate(prompts, max_new_tokens=5)
        out["first_token_match"] = [a[0] == b[0] for a, b in zip(tp_out, ref_out)]
        pairs = [(x, y) for a, b in zip(tp_out, ref_out) for x, y in zip(a, b)]
        out["token_match_rate"] = sum(x == y for x, y in pairs) / len(pairs)
        out["tp_tokens"] = tp_out
        out["ref_tokens"] = ref_out
    ops.check_status()
    dist.barrier()
    if rank == 0:
        print("TPJSON " + json.dumps(out))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
