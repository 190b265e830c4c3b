"""Checked indices: every kernel that takes an index from its caller (a KV
page-copy pair, a token's cache slot, a token id, a block-table page)
verifies it before the access. An index outside its pool is never used: the
access is skipped (or reads an out-of-range, zero-filled TMA box), the
first fault is recorded in the status words (code 7, site, index) and the
rest of the launch completes normally."""
import math

import numpy as np
import pytest
import torch

from sched_pass_b200 import ops
from sched_pass_b200._ext import ext
from sched_pass_b200.models import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def expect_bad_index(site, index):
    with pytest.raises(ops.KernelStatusError) as e:
        ops.check_status()
    assert (e.value.code, e.value.site, e.value.index) == (7, site, index), str(e.value)
    ops.check_status()  # cleared


@pytest.fixture(autouse=True)
def _clean():
    ops.check_status()
    yield


def test_page_copy_skips_pairs_outside_the_pools():
    L, N, H = 2, 6, 2
    k = torch.randn(L, N, H, 16, 128, device=DEV).to(torch.bfloat16)
    v = torch.randn_like(k)
    dk = torch.zeros(L, 4, H, 16, 128, dtype=torch.bfloat16, device=DEV)
    dv = torch.zeros_like(dk)
    pairs = torch.tensor([[1, 0], [99, 1], [2, 3]], dtype=torch.int32, device=DEV)
    ext().kv_page_copy(k, v, dk, dv, pairs, 3, None, ops.status_buffer())
    torch.cuda.synchronize()
    assert torch.equal(dk[:, 0], k[:, 1]) and torch.equal(dk[:, 3], k[:, 2])
    assert dk[:, 1].abs().sum().item() == 0
    expect_bad_index(1, 99)
    pairs = torch.tensor([[0, 4]], dtype=torch.int32, device=DEV)  # destination pool has 4 pages
    ext().kv_page_copy(k, v, dk, dv, pairs, 1, None, ops.status_buffer())
    torch.cuda.synchronize()
    expect_bad_index(2, 4)


def test_fp8_page_copy_skips_pairs_outside_the_pools():
    L, N, H = 1, 3, 1
    k = torch.randn(L, N, H, 16, 128, device=DEV).to(torch.bfloat16)
    hk = torch.zeros(L, 2, H, 16, 128, dtype=torch.uint8, device=DEV)
    hv = torch.zeros_like(hk)
    sk = torch.zeros(L, 2, H, dtype=torch.float32, device=DEV)
    sv = torch.zeros_like(sk)
    pairs = torch.tensor([[0, 1], [1, -3]], dtype=torch.int32, device=DEV)
    ext().kv_page_copy_fp8(k, k, hk, hv, sk, sv, True, pairs, 2, None, ops.status_buffer())
    torch.cuda.synchronize()
    assert sk[0, 1, 0].item() > 0 and sk[0, 0, 0].item() == 0
    expect_bad_index(2, -3)


def test_kv_append_skips_slots_outside_the_cache():
    from sched_pass_b200.models.config import LLAMA_TINY
    from sched_pass_b200.models.llama import rope_table
    cfg = LLAMA_TINY
    T, Hq, Hkv, D = 3, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    cs = rope_table(cfg, 64, DEV)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=DEV).to(torch.bfloat16)
    pos = torch.tensor([0, 1, 2], dtype=torch.int32, device=DEV)
    slot = torch.tensor([3, 8 * 16 + 5, 17], dtype=torch.int32, device=DEV)  # cache of 8 pages
    kc = torch.zeros(8, Hkv, 16, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=DEV)
    ops.rope_kv_append(qkv, pos, slot, cs, q, kc, vc, Hq, Hkv)
    torch.cuda.synchronize()
    v = qkv.view(T, Hq + 2 * Hkv, D)
    assert torch.equal(vc[0, :, 3], v[0, Hq + Hkv:]) and torch.equal(vc[1, :, 1], v[2, Hq + Hkv:])
    assert int((vc.abs().sum(dim=(1, 3)) > 0).sum()) == 2  # only the two valid slots written
    expect_bad_index(3, 8 * 16 + 5)


def test_fused_qkv_rope_epilogue_skips_slots_outside_the_cache():
    from sched_pass_b200.models.config import LLAMA_TINY
    from sched_pass_b200.models.llama import rope_table
    cfg = LLAMA_TINY
    T, Hq, Hkv, D, K = 4, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, 256
    x = torch.randn(T, K, device=DEV).to(torch.bfloat16)
    w = (torch.randn((Hq + 2 * Hkv) * D, K, device=DEV) / 16).to(torch.bfloat16)
    cs = rope_table(cfg, 64, DEV)
    pos = torch.arange(T, dtype=torch.int32, device=DEV)
    slot = torch.tensor([0, 1, 4 * 16, 2], dtype=torch.int32, device=DEV)  # cache of 4 pages
    kc = torch.zeros(4, Hkv, 16, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=DEV)
    ops.linear_qkv_rope(x, w, pos, slot, cs, q, kc, vc, Hq, Hkv)
    torch.cuda.synchronize()
    assert int((vc[0].abs().sum(dim=(0, 2)) > 0).sum()) == 3 and vc[1:].abs().sum().item() == 0
    expect_bad_index(3, 4 * 16)


def test_embedding_zeroes_rows_of_ids_outside_the_vocabulary():
    table = torch.randn(100, 256, device=DEV).to(torch.bfloat16)
    ids = torch.tensor([3, 100, 7], dtype=torch.int32, device=DEV)
    out = ops.embedding(ids, table)
    torch.cuda.synchronize()
    assert torch.equal(out[0], table[3]) and torch.equal(out[2], table[7]) and out[1].abs().sum().item() == 0
    expect_bad_index(4, 100)


def test_decode_reads_a_bad_page_as_zeros_and_reports_it():
    from sched_pass_b200.engine import native
    Hkv, G, D = 2, 4, 128
    lens = [40, 70]
    P = 12
    g = torch.Generator().manual_seed(3)
    kc = torch.randn(P, Hkv, 16, D, generator=g).to(torch.bfloat16).to(DEV)
    vc = torch.randn(P, Hkv, 16, D, generator=g).to(torch.bfloat16).to(DEV)
    bt = torch.tensor([[0, 1, 2, 0, 0], [3, 4, 500, 5, 6]], dtype=torch.int32, device=DEV)
    q = torch.randn(2, Hkv * G, D, device=DEV).to(torch.bfloat16)
    items, _, _ = native.plan_decode(np.asarray(lens, dtype=np.int32), 1)
    out = torch.zeros_like(q)
    ops.attention_decode(q, out, kc, vc, bt, torch.from_numpy(items).to(DEV), items.shape[0], 1 / math.sqrt(D),
                         woven=False)
    torch.cuda.synchronize()
    # reference: page 500 replaced by an all-zero page
    kz = torch.cat([kc, torch.zeros(1, Hkv, 16, D, dtype=kc.dtype, device=DEV)])
    vz = torch.cat([vc, torch.zeros(1, Hkv, 16, D, dtype=vc.dtype, device=DEV)])
    bt_ref = bt.clone()
    bt_ref[1, 2] = P
    r = ref.decode_attention_paged(q, kz, vz, bt_ref, lens, 1 / math.sqrt(D))
    assert ((out.float() - r.float()).norm() / r.float().norm()).item() < 2e-2
    expect_bad_index(5, 500)
