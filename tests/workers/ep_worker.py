"""torchrun worker: one MoE layer with experts split across ranks (fused
NVLink dispatch / expert GEMM / combine) vs an fp32 oracle over all experts."""
import faulthandler
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

from sched_pass_b200 import ops  # noqa: E402
from sched_pass_b200.models import reference as ref  # noqa: E402
from sched_pass_b200.models.config import MIXTRAL_TINY  # noqa: E402
from sched_pass_b200.parallel.ep import ExpertParallel, build_moe_weights, dequantize_blockwise_fp8  # noqa: E402
from sched_pass_b200.parallel.tp import init_distributed  # noqa: E402


def quant_rows(x):
    T, H = x.shape
    xb = x.reshape(T, H // 128, 128)
    s = (xb.abs().amax(-1, keepdim=True) / 448.0).clamp_min(1e-30)
    return ((xb / s).to(torch.float8_e4m3fn).float() * s).reshape(T, H)


def gather(t):
    ts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(ts, t)
    return torch.cat(ts)


faulthandler.enable()  # a native crash prints the Python stack of every thread


def main():
    rank, world, local = init_distributed("nccl", timeout_s=60)
    dev = torch.device("cuda", local)
    cfg = MIXTRAL_TINY
    E, H, I = cfg.n_experts, cfg.hidden, cfg.ffn
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    w = build_moe_weights(cfg, rank, world, g, dev)
    w13 = gather(w.w13.view(torch.uint8)).view(torch.float8_e4m3fn)
    s13 = gather(w.s13)
    w2 = gather(w.w2.view(torch.uint8)).view(torch.float8_e4m3fn)
    s2 = gather(w.s2)
    w13e = [dequantize_blockwise_fp8(w13[e * 2 * I:(e + 1) * 2 * I], s13[e]) for e in range(E)]
    w2e = [dequantize_blockwise_fp8(w2[e * H:(e + 1) * H], s2[e]) for e in range(E)]
    ep = ExpertParallel(cfg, dev, max_tokens=64)
    out = {"checks": []}
    ln = torch.ones(H, dtype=torch.bfloat16, device=dev)
    # per-rank token counts, including a rank with none (it must still serve its experts)
    for case in ([5, 12], [0, 33], [64, 1], [17, 0]):
        T = case[rank % 2]
        gx = torch.Generator(device=dev).manual_seed(7 * rank + len(out["checks"]))
        x = torch.randn(T, H, device=dev, generator=gx).to(torch.bfloat16)
        h0 = torch.randn(T, H, device=dev, generator=gx).to(torch.bfloat16)
        h = h0.clone()
        y = torch.empty_like(x)
        errs = []
        for rep in range(3):
            h.copy_(h0)
            ep.layer(w, x, h, ln, y, cfg.rms_eps)
            torch.cuda.synchronize()
            if T:
                delta, _, _ = ref.moe(x, w.router, w13e, w2e, cfg.top_k, quantize_x=quant_rows,
                                      quantize_act=quant_rows)
                got = h.float() - h0.float()
                errs.append(((got - delta).norm() / delta.norm()).item())
        out["checks"].append({"rank": rank, "T": T, "rel_err": max(errs) if errs else 0.0})
    ops.check_status()
    out["dropped"] = ep.dropped_total()
    allc = [None] * world
    dist.all_gather_object(allc, out)
    ep.close()
    dist.barrier()
    if rank == 0:
        print("EPJSON " + json.dumps(allc))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
