"""MoE layer on one GPU (all experts local): router, dispatch, tcgen05 fp8
block-scaled expert GEMMs, combine + residual + RMSNorm vs an fp32 oracle."""
import math

import pytest
import torch

from sched_pass_b200 import ops
from sched_pass_b200._ext import ext
from sched_pass_b200.models import reference as ref
from sched_pass_b200.models.config import MIXTRAL_TINY
from sched_pass_b200.parallel.ep import ExpertParallel, build_moe_weights, dequantize_blockwise_fp8

pytestmark = pytest.mark.gpu


def quant_rows(x):
    """The dispatch's activation quantisation: e4m3 with a scale per 128 columns."""
    T, H = x.shape
    xb = x.reshape(T, H // 128, 128)
    s = (xb.abs().amax(-1, keepdim=True) / 448.0).clamp_min(1e-30)
    return ((xb / s).to(torch.float8_e4m3fn).float() * s).reshape(T, H)


def setup(T, capacity=None, seed=0):
    cfg = MIXTRAL_TINY
    ep = ExpertParallel(cfg, "cuda", max_tokens=64, capacity=capacity)
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = build_moe_weights(cfg, 0, 1, g, "cuda")
    x = torch.randn(T, cfg.hidden, device="cuda", generator=g).to(torch.bfloat16)
    h = torch.randn(T, cfg.hidden, device="cuda", generator=g).to(torch.bfloat16)
    ln = torch.ones(cfg.hidden, dtype=torch.bfloat16, device="cuda")
    return cfg, ep, w, x, h, ln


def experts(cfg, w):
    E, H, I = cfg.n_experts, cfg.hidden, cfg.ffn
    w13 = [dequantize_blockwise_fp8(w.w13[e * 2 * I:(e + 1) * 2 * I].view(torch.float8_e4m3fn), w.s13[e]) for e in range(E)]
    w2 = [dequantize_blockwise_fp8(w.w2[e * H:(e + 1) * H].view(torch.float8_e4m3fn), w.s2[e]) for e in range(E)]
    return w13, w2


@pytest.mark.parametrize("T", [1, 7, 33])
def test_moe_layer_matches_reference(T):
    cfg, ep, w, x, h, ln = setup(T)
    h0 = h.clone()
    y = torch.empty_like(x)
    for rep in range(3):  # counters must reset themselves between layers
        h.copy_(h0)
        ep.layer(w, x, h, ln, y, cfg.rms_eps)
        torch.cuda.synchronize()
        ops.check_status()
        w13, w2 = experts(cfg, w)
        delta, _, _ = ref.moe(x, w.router, w13, w2, cfg.top_k, quantize_x=quant_rows, quantize_act=quant_rows)
        got = h.float() - h0.float()
        err = ((got - delta).norm() / delta.norm()).item()
        assert err < 3e-2, err
        assert ((y.float() - ref.rmsnorm(h, ln, cfg.rms_eps)).norm() / y.float().norm()).item() < 1e-2
    assert ep.dropped_total() == 0


def test_moe_capacity_drops_overflow():
    T = 40
    cfg, ep, w, x, h, ln = setup(T, capacity=8, seed=3)
    ids = torch.empty(T, cfg.top_k, dtype=torch.int32, device="cuda")
    wts = torch.empty(T, cfg.top_k, dtype=torch.float32, device="cuda")
    ext().moe_router(x, w.router, ids, wts, cfg.top_k)
    counts = torch.bincount(ids.reshape(-1).long(), minlength=cfg.n_experts)
    expect = int((counts - 8).clamp_min(0).sum())
    y = torch.empty_like(x)
    ep.layer(w, x, h, ln, y, cfg.rms_eps)
    torch.cuda.synchronize()
    ops.check_status()
    assert ep.dropped_total() == expect and expect > 0


def test_mixtral_engine_generates_like_reference():
    import numpy as np

    from sched_pass_b200.engine.engine import Engine, EngineConfig
    from sched_pass_b200.models.llama import rope_table
    from sched_pass_b200.models.mixtral import mixtral_factory

    cfg = MIXTRAL_TINY
    ecfg = EngineConfig(max_batch=8, max_prefill_tokens=128, max_context=256)
    T = max(ecfg.max_prefill_tokens + ecfg.max_batch, 256)
    ep = ExpertParallel(cfg, "cuda", max_tokens=T)
    eng = Engine(cfg, ecfg, "cuda", model_factory=mixtral_factory(ep, 0, 1))
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, cfg.vocab, size=int(n)).astype(np.int32) for n in (5, 40, 17)]
    out = eng.generate(prompts, max_new_tokens=4)
    ops.check_status()
    assert all(len(o) == 4 for o in out)
    cos_sin = rope_table(cfg, 512, "cuda")

    def experts_of(lw):
        return experts(cfg, lw.moe)

    for p, o in zip(prompts, out):
        logits = ref.mixtral_forward_tokens(cfg, eng.model.w, p, cos_sin, experts_of, quantize=quant_rows)
        top2 = logits.topk(2).values
        if (top2[0] - top2[1]).item() > 0.05:  # skip near-ties
            assert int(logits.argmax()) == o[0]
    assert ep.dropped_total() == 0
    ep.close()
