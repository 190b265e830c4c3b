"""Plain-PyTorch fp32 statements of every kernel, used as test oracles.

These are definitions, not a fallback: nothing in the serving path calls
them. Each mirrors one native kernel's contract exactly (layouts included).
"""
from __future__ import annotations

import math

import torch


def linear(x, w):
    return x.float() @ w.float().t()


def swiglu_linear(x, w_interleaved, block: int = 64):
    y = linear(x, w_interleaved)
    T, N2 = y.shape
    v = y.reshape(T, N2 // (2 * block), 2, block)
    g, u = v[:, :, 0].reshape(T, -1), v[:, :, 1].reshape(T, -1)
    return torch.nn.functional.silu(g) * u


def rmsnorm(x, w, eps):
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def rope(x, pos, cos_sin):
    """Rotate-half RoPE. x [T, H, D]; cos_sin [max_pos, D/2, 2]."""
    D = x.shape[-1]
    half = D // 2
    cs = cos_sin[pos.long()]  # [T, D/2, 2]
    c, s = cs[..., 0][:, None, :], cs[..., 1][:, None, :]
    a, b = x[..., :half].float(), x[..., half:].float()
    return torch.cat([a * c - b * s, b * c + a * s], dim=-1)


def gather_kv(cache, block_table_row, n_tokens, page_size=16):
    """cache [pages, Hkv, 16, D] -> [n_tokens, Hkv, D] for one request."""
    pages = block_table_row[: (n_tokens + page_size - 1) // page_size].long()
    kv = cache[pages]                      # [np, Hkv, 16, D]
    kv = kv.permute(0, 2, 1, 3).reshape(-1, cache.shape[1], cache.shape[3])
    return kv[:n_tokens]


def attention(q, k, v, sm_scale, causal_offset=None, tau=0):
    """q [Tq, Hq, D]; k, v [Tk, Hkv, D]. GQA by head grouping. With
    ``causal_offset`` c, query i sees keys [0, c + i]. ``tau`` > 0 keeps only
    keys with index < tau (exact truncated softmax)."""
    Tq, Hq, D = q.shape
    Tk, Hkv, _ = k.shape
    G = Hq // Hkv
    kf = k.float().repeat_interleave(G, dim=1)
    vf = v.float().repeat_interleave(G, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kf) * sm_scale
    mask = torch.zeros(Tq, Tk, dtype=torch.bool, device=q.device)
    if causal_offset is not None:
        qi = torch.arange(Tq, device=q.device)[:, None] + causal_offset
        ki = torch.arange(Tk, device=q.device)[None, :]
        mask |= ki > qi
    if tau > 0:
        mask |= torch.arange(Tk, device=q.device)[None, :] >= tau
    s = s.masked_fill(mask[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    return torch.einsum("hqk,khd->qhd", p, vf)


def decode_attention_paged(q, k_cache, v_cache, block_table, seq_lens, sm_scale, taus=None):
    """q [B, Hq, D]; one query token per request, attending to its first
    seq_lens[b] tokens (or the first tau when tau > 0)."""
    outs = []
    for b in range(q.shape[0]):
        n = int(seq_lens[b])
        k = gather_kv(k_cache, block_table[b], n)
        v = gather_kv(v_cache, block_table[b], n)
        tau = int(taus[b]) if taus is not None else 0
        outs.append(attention(q[b:b + 1], k, v, sm_scale, tau=tau)[0])
    return torch.stack(outs)


def llama_forward_tokens(cfg, weights, token_ids, cos_sin):
    """Greedy-free reference forward of ONE sequence from scratch (all tokens
    in one prefill): returns fp32 logits of the last position. Single rank."""
    dev = weights.embed.device
    ids = torch.as_tensor(token_ids, dtype=torch.long, device=dev)
    T = ids.numel()
    pos = torch.arange(T, device=dev)
    h = weights.embed[ids].float()
    D = cfg.head_dim
    for li, lw in enumerate(weights.layers):
        x = rmsnorm(h, lw.ln_in, cfg.rms_eps).to(torch.bfloat16)
        qkv = linear(x, lw.qkv)
        hq = lw.o.shape[1] // D
        hkv = (lw.qkv.shape[0] // D - hq) // 2
        q = qkv[:, : hq * D].reshape(T, hq, D)
        k = qkv[:, hq * D:(hq + hkv) * D].reshape(T, hkv, D)
        v = qkv[:, (hq + hkv) * D:].reshape(T, hkv, D)
        q = rope(q.to(torch.bfloat16), pos, cos_sin).to(torch.bfloat16)
        k = rope(k.to(torch.bfloat16), pos, cos_sin).to(torch.bfloat16)
        a = attention(q, k, v.to(torch.bfloat16), 1.0 / math.sqrt(D), causal_offset=0)
        o = linear(a.reshape(T, -1).to(torch.bfloat16), lw.o)
        h = (h + o.to(torch.bfloat16).float()).to(torch.bfloat16).float()
        x = rmsnorm(h, lw.ln_post, cfg.rms_eps).to(torch.bfloat16)
        act = swiglu_linear(x, lw.gate_up).to(torch.bfloat16)
        d = linear(act, lw.down)
        h = (h + d.to(torch.bfloat16).float()).to(torch.bfloat16).float()
    x = rmsnorm(h, weights.ln_final, cfg.rms_eps).to(torch.bfloat16)
    return linear(x[-1:], weights.lm_head)[0, : cfg.vocab]


def moe(x, router, w13_experts, w2_experts, top_k, block=64, quantize_x=None, quantize_act=None):
    """Top-k softmax-routed SwiGLU experts. w13_experts[e]: [2I, H] with
    gate/up interleaved per ``block`` rows; w2_experts[e]: [H, I]; all fp32.
    ``quantize_x(x) -> x'`` / ``quantize_act(a) -> a'`` optionally apply the
    kernels' quantisation of the token rows and of the SwiGLU output."""
    xf = x.float()
    logits = xf @ router.float().t()
    val, idx = logits.topk(top_k, dim=-1)
    wts = torch.softmax(val, dim=-1)
    xq = quantize_x(xf) if quantize_x is not None else xf
    out = torch.zeros_like(xf)
    for t in range(xf.shape[0]):
        for j in range(top_k):
            e = int(idx[t, j])
            y = swiglu_linear(xq[t:t + 1], w13_experts[e], block)
            y = y.to(torch.bfloat16).float()
            if quantize_act is not None:
                y = quantize_act(y)
            out[t] += wts[t, j] * (y @ w2_experts[e].float().t())[0]
    return out, idx, wts


def mixtral_forward_tokens(cfg, weights, token_ids, cos_sin, experts_of, quantize=None):
    """``llama_forward_tokens`` with the FFN replaced by top-k MoE.
    ``experts_of(layer_weights) -> (w13 list, w2 list)`` gives fp32 expert
    weights; ``quantize`` is applied to expert inputs and SwiGLU outputs."""
    dev = weights.embed.device
    ids = torch.as_tensor(token_ids, dtype=torch.long, device=dev)
    T = ids.numel()
    pos = torch.arange(T, device=dev)
    h = weights.embed[ids].float()
    D = cfg.head_dim
    for lw in weights.layers:
        x = rmsnorm(h, lw.ln_in, cfg.rms_eps).to(torch.bfloat16)
        qkv = linear(x, lw.qkv)
        hq = lw.o.shape[1] // D
        hkv = (lw.qkv.shape[0] // D - hq) // 2
        q = qkv[:, : hq * D].reshape(T, hq, D)
        k = qkv[:, hq * D:(hq + hkv) * D].reshape(T, hkv, D)
        v = qkv[:, (hq + hkv) * D:].reshape(T, hkv, D)
        q = rope(q.to(torch.bfloat16), pos, cos_sin).to(torch.bfloat16)
        k = rope(k.to(torch.bfloat16), pos, cos_sin).to(torch.bfloat16)
        a = attention(q, k, v.to(torch.bfloat16), 1.0 / math.sqrt(D), causal_offset=0)
        o = linear(a.reshape(T, -1).to(torch.bfloat16), lw.o)
        h = (h + o.to(torch.bfloat16).float()).to(torch.bfloat16).float()
        x = rmsnorm(h, lw.ln_post, cfg.rms_eps).to(torch.bfloat16)
        w13, w2 = experts_of(lw)
        d, _, _ = moe(x, lw.moe.router, w13, w2, cfg.top_k, quantize_x=quantize, quantize_act=quantize)
        h = (h + d).to(torch.bfloat16).float()
    x = rmsnorm(h, weights.ln_final, cfg.rms_eps).to(torch.bfloat16)
    return linear(x[-1:], weights.lm_head)[0, : cfg.vocab]
