"""End-to-end engine checks on a small Llama-architecture model."""
import numpy as np
import pytest
import torch

from sched_pass_b200 import ops
from sched_pass_b200.engine.engine import Engine, EngineConfig
from sched_pass_b200.models import reference as ref
from sched_pass_b200.models.config import LLAMA_TINY
from sched_pass_b200.models.llama import init_weights, rope_table

pytestmark = pytest.mark.gpu


def prompts(n, lo=5, hi=300, seed=0):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, LLAMA_TINY.vocab, size=int(rng.integers(lo, hi))).astype(np.int32)
            for _ in range(n)]


def make_engine(**kw):
    cfg = LLAMA_TINY
    e = EngineConfig(max_batch=16, max_prefill_tokens=512, max_context=1024, **kw)
    w = init_weights(cfg, "cuda", seed=3)
    return Engine(cfg, e, "cuda", weights=w), w


def test_engine_greedy_tracks_reference():
    eng, w = make_engine(cuda_graphs=False)
    ps = prompts(3, seed=1)
    outs = eng.generate(ps, max_new_tokens=4)
    ops.check_status()
    cs = rope_table(LLAMA_TINY, 2048, "cuda")
    for p, o in zip(ps, outs):
        seq = list(p)
        for tok in o:
            logits = ref.llama_forward_tokens(LLAMA_TINY, w, seq, cs)
            top = logits.max().item()
            spread = logits.std().item()
            assert logits[tok].item() >= top - 0.05 * spread, "engine token far from reference argmax"
            seq.append(tok)


def test_graphs_and_levers_do_not_change_tokens():
    ps = prompts(6, seed=2)
    base, _ = make_engine(cuda_graphs=False, levers=False)
    ref_out = base.generate(ps, max_new_tokens=6)
    del base
    for kw in (dict(cuda_graphs=True, levers=False), dict(cuda_graphs=True, levers=True),
               dict(cuda_graphs=True, levers=True, acquire="clc"),
               dict(cuda_graphs=False, levers=True, acquire="ticket")):
        eng, _ = make_engine(**kw)
        assert eng.generate(ps, max_new_tokens=6) == ref_out, kw
        ops.check_status()
        del eng
        torch.cuda.empty_cache()


def test_chunked_prefill_and_preemption():
    eng, _ = make_engine(cuda_graphs=True)
    eng.ecfg.max_prefill_tokens = 64  # force several prefill chunks per prompt
    eng.sched.max_prefill_tokens = 64
    ps = prompts(5, lo=100, hi=200, seed=4)
    outs = eng.generate(ps, max_new_tokens=3)
    assert all(len(o) == 3 for o in outs)
    assert eng.sched.alloc.free == eng.sched.alloc.num_pages


def test_capped_mixed_steps_replay_graphs_with_the_eager_tokens():
    """With a per-step token cap, mixed decode + prefill steps are padded to a
    fixed shape per decode bucket and replayed from CUDA graphs; the padded
    eager run of the same steps produces the same tokens, every step stays
    within the cap (counting padded decode rows), and graphs serve the mixed
    steps."""
    ps = prompts(10, lo=40, hi=400, seed=7)
    runs = {}
    for graphs in (False, True):
        eng, _ = make_engine(cuda_graphs=graphs, max_step_tokens=96)
        runs[graphs] = eng.generate(ps, max_new_tokens=8)
        ops.check_status()
        mixed = [s for s in eng.stats if s.n_prefill_tokens > 0 and s.n_decode > 0]
        assert mixed, "no mixed steps"
        assert all(s.n_prefill_tokens <= 96 for s in eng.stats)
        if graphs:
            assert sum(s.graph for s in mixed) >= len(mixed) // 2, [(s.n_decode, s.graph) for s in mixed]
        assert eng.sched.alloc.free == eng.sched.alloc.num_pages
        eng.graphs.clear()
        del eng
        torch.cuda.empty_cache()
    assert runs[True] == runs[False]


def test_prefill_tile_order_does_not_change_tokens():
    """Longest-first prefill tiles (the default) and plan order give the
    same tokens: each tile writes only its own rows."""
    ps = prompts(5, lo=100, hi=400, seed=9)
    outs = []
    for order in ("identity", "lpt"):
        eng, _ = make_engine(cuda_graphs=True, prefill_order=order)
        outs.append(eng.generate(ps, max_new_tokens=4))
        ops.check_status()
        eng.graphs.clear()
        del eng
        torch.cuda.empty_cache()
    assert outs[0] == outs[1]


def _generate_sync(eng, ps, n):
    """The same requests as ``Engine.generate`` but one synchronous step at a time."""
    from sched_pass_b200.engine.request import Request
    reqs = [Request(rid=i, prompt=np.asarray(p, dtype=np.int32), max_new_tokens=n) for i, p in enumerate(ps)]
    for r in reqs:
        eng.add_request(r)
    while eng.has_work():
        eng.step()
    return reqs


def test_async_steps_match_synchronous_steps():
    """The host planning step k + 1 while the device runs step k (decode
    inputs taken from the previous step's sampled ids on the device) gives
    the same tokens as reading every step back before planning the next;
    every token time is filled in and the same number of steps ran. Also
    under preemption (a KV pool too small for every request at once), where
    pending tokens are read back before a request's output joins its prompt."""
    ps = prompts(8, lo=20, hi=260, seed=11)
    for kw in (dict(cuda_graphs=True, levers=True), dict(cuda_graphs=False, levers=True, acquire="clc"),
               dict(cuda_graphs=True, levers=True, num_pages=48)):
        a, _ = make_engine(**kw)
        want = _generate_sync(a, ps, 7)
        n_sync = len(a.stats)
        a.graphs.clear()
        del a
        b, _ = make_engine(**kw)
        got = b.generate(ps, max_new_tokens=7)
        ops.check_status()
        assert got == [r.output for r in want], kw
        assert len(b.stats) == n_sync, kw
        assert b.sched.alloc.free == b.sched.alloc.num_pages
        b.graphs.clear()
        del b
        torch.cuda.empty_cache()
    for r in want:
        assert all(np.isfinite(r.token_times)) and r.token_times == sorted(r.token_times)
