"""Tiered KV on the GPU: the page-copy kernel between device and pinned
host pools, and an engine whose device pool is too small for its requests
(pages spill to host and are staged back every step) generating exactly the
tokens of an engine that keeps everything on the device."""
import numpy as np
import pytest
import torch

from sched_pass_b200 import ops
from sched_pass_b200._ext import ext

pytestmark = pytest.mark.gpu


def test_page_copy_roundtrip_through_pinned_host():
    L, N, H = 3, 10, 2
    k = torch.randn(L, N, H, 16, 128, device="cuda").to(torch.bfloat16)
    v = torch.randn_like(k)
    hk = torch.zeros(L, 6, H, 16, 128, dtype=torch.bfloat16, pin_memory=True)
    hv = torch.zeros_like(hk, pin_memory=True)
    pairs = torch.tensor([[7, 0], [2, 5], [9, 3]], dtype=torch.int32, device="cuda")
    ext().kv_page_copy(k, v, hk, hv, pairs, 3, None, None)
    torch.cuda.synchronize()
    for s, d in ((7, 0), (2, 5), (9, 3)):
        assert torch.equal(hk[:, d], k[:, s].cpu()) and torch.equal(hv[:, d], v[:, s].cpu())
    k2, v2 = torch.zeros_like(k), torch.zeros_like(v)
    back = torch.tensor([[0, 1], [5, 4], [3, 8]], dtype=torch.int32, device="cuda")
    ext().kv_page_copy(hk, hv, k2, v2, back, 3, None, None)
    torch.cuda.synchronize()
    assert torch.equal(k2[:, 1], k[:, 7]) and torch.equal(v2[:, 8], v[:, 9])


def test_engine_with_spilled_kv_matches_device_only_engine():
    from sched_pass_b200.engine.engine import Engine, EngineConfig
    from sched_pass_b200.engine.request import Request
    from sched_pass_b200.models.config import LLAMA_TINY
    from sched_pass_b200.models.llama import full_weights, shard_weights
    cfg = LLAMA_TINY
    full = full_weights(cfg, seed=11)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, cfg.vocab, size=n).astype(np.int32) for n in (150, 90, 200, 120)]
    urg = [0.9, 0.1, 0.5, 0.3]

    def run(**kw):
        eng = Engine(cfg, EngineConfig(max_batch=8, max_prefill_tokens=256, max_context=512, **kw), "cuda",
                     weights=shard_weights(cfg, full, 0, 1, "cuda"))
        reqs = [Request(rid=i, prompt=p, max_new_tokens=24, urgency=u) for i, (p, u) in enumerate(zip(prompts, urg))]
        for r in reqs:
            eng.add_request(r)
        while eng.has_work():
            eng.step()
        ops.check_status()
        return [r.output for r in reqs], eng, reqs

    ref, _, _ = run()
    # the copy engines (cudaMemcpyAsync per run of host pages) and the
    # zero-copy kernel stage the same bytes
    for mode in ("copy", "kernel"):
        got, eng, reqs = run(num_pages=30, host_kv_pages=64, kv_staging_pages=40, kv_stage_mode=mode)
        assert eng.tier.stage_mode == mode
        assert eng.tier.spilled_pages > 0 and eng.tier.staged_pages > 0
        assert got == ref, mode
        assert all(r.preemptions == 0 for r in reqs)  # spilling replaced preemption


def _fp8_reference(x):
    """fp32 reference of the fp8 page quantization: per (layer, page, head)
    scale = amax / 448, q = e4m3(x * (1 / scale)), x' = q * scale."""
    xf = x.float()
    amax = xf.abs().amax(dim=(-2, -1), keepdim=True)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (xf * (1.0 / scale)).to(torch.float8_e4m3fn)
    return q, scale, (q.float() * scale).to(torch.bfloat16)


def test_fp8_page_copy_matches_fp32_reference():
    L, N, H = 2, 9, 3
    k = (torch.randn(L, N, H, 16, 128, device="cuda") * 3).to(torch.bfloat16)
    v = (torch.randn_like(k, dtype=torch.float32) * 0.01).to(torch.bfloat16)
    k[1, 4].zero_()  # an all-zero page keeps scale 1
    hk = torch.zeros(L, 5, H, 16, 128, dtype=torch.uint8, pin_memory=True)
    hv = torch.zeros_like(hk, pin_memory=True)
    sk = torch.zeros(L, 5, H, dtype=torch.float32, pin_memory=True)
    sv = torch.zeros_like(sk, pin_memory=True)
    pairs = torch.tensor([[7, 0], [4, 3], [1, 4]], dtype=torch.int32, device="cuda")
    ext().kv_page_copy_fp8(k, v, hk, hv, sk, sv, True, pairs, 3, None, None)
    torch.cuda.synchronize()
    for s, d in ((7, 0), (4, 3), (1, 4)):
        for x, hq, hs in ((k, hk, sk), (v, hv, sv)):
            q, scale, _ = _fp8_reference(x[:, s].cpu())
            torch.testing.assert_close(hs[:, d], scale.reshape(L, H), rtol=0, atol=0)
            same = (hq[:, d] == q.view(torch.uint8)).float().mean().item()
            assert same > 0.999, same  # bit-identical except rare rounding-tie differences
    # fetch back through the dequantizing copy into a bf16 pool
    k2, v2 = torch.zeros_like(k), torch.zeros_like(v)
    back = torch.tensor([[0, 2], [3, 5], [4, 8]], dtype=torch.int32, device="cuda")
    ext().kv_page_copy_fp8(hk, hv, k2, v2, sk, sv, False, back, 3, None, None)
    torch.cuda.synchronize()
    for s, d in ((7, 2), (4, 5), (1, 8)):
        for x, y in ((k, k2), (v, v2)):
            _, _, ref = _fp8_reference(x[:, s].cpu())
            torch.testing.assert_close(y[:, d].cpu().float(), ref.float(), rtol=0.02, atol=1e-6)
            err = (y[:, d].float() - x[:, s].float()).abs().max() / x[:, s].float().abs().max().clamp_min(1e-6)
            assert err.item() < 0.07  # e4m3 keeps 3 mantissa bits


def test_engine_with_fp8_host_tier_tracks_device_only_engine():
    """With an fp8 host pool the spilled pages come back at fp8 precision:
    the run completes without preemption, requests that never spilled
    generate exactly the all-device engine's tokens (attention is per
    request), and the spilled ones finish their budget."""
    from sched_pass_b200.engine.engine import Engine, EngineConfig
    from sched_pass_b200.engine.request import Request
    from sched_pass_b200.models.config import LLAMA_TINY
    from sched_pass_b200.models.llama import full_weights, shard_weights
    cfg = LLAMA_TINY
    full = full_weights(cfg, seed=11)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, cfg.vocab, size=n).astype(np.int32) for n in (150, 90, 200, 120)]
    urg = [0.9, 0.1, 0.5, 0.3]

    def run(**kw):
        eng = Engine(cfg, EngineConfig(max_batch=8, max_prefill_tokens=256, max_context=512, **kw), "cuda",
                     weights=shard_weights(cfg, full, 0, 1, "cuda"))
        reqs = [Request(rid=i, prompt=p, max_new_tokens=24, urgency=u) for i, (p, u) in enumerate(zip(prompts, urg))]
        for r in reqs:
            eng.add_request(r)
        while eng.has_work():
            eng.step()
        ops.check_status()
        return reqs, eng

    ref, _ = run()
    got, eng = run(num_pages=30, host_kv_pages=64, kv_staging_pages=40, host_kv_dtype="fp8")
    assert eng.tier.spilled_pages > 0 and eng.tier.staged_pages > 0
    assert all(r.preemptions == 0 and len(r.output) == 24 for r in got)
    spilled = [r.spilled_pages > 0 for r in got]
    assert any(spilled) and not all(spilled)
    for x, y in zip(ref, got):
        if y.spilled_pages == 0:
            assert x.output == y.output
