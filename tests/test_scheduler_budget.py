"""The scheduler's per-step token cap (stall-free batching): decode +
prefill tokens of a step stay within ``max_step_tokens`` while prefill still
progresses when the decode batch alone fills the cap; without the cap the
old behaviour (prefill chunks up to ``max_prefill_tokens``) is unchanged.
CPU only (the native page allocator)."""
import numpy as np

from sched_pass_b200.engine.request import Request
from sched_pass_b200.engine.scheduler import Scheduler


def drive(sched, reqs, arrivals_per_step=1, steps=4000):
    """Fake model: every produced token is 1. Returns the per-step plans'
    (n_decode, n_prefill) and the finished requests."""
    pending = list(reqs)
    shapes, done = [], []
    for step in range(steps):
        for _ in range(arrivals_per_step):
            if pending:
                sched.add(pending.pop(0))
        if sched.idle and not pending:
            break
        plan = sched.schedule()
        sampled = {r.rid: 1 for r in plan.decode}
        for r, start, n in plan.prefill:
            if start + n >= r.prompt_len:
                sampled[r.rid] = 1
        shapes.append((len(plan.decode), sum(n for _, _, n in plan.prefill)))
        done += sched.commit(plan, sampled, float(step))
    return shapes, done


def make(n, prompt=1536, out=32, seed=0):
    rng = np.random.default_rng(seed)
    return [Request(rid=i, prompt=rng.integers(0, 1000, size=prompt).astype(np.int32), max_new_tokens=out)
            for i in range(n)]


def test_step_cap_bounds_every_step_and_everything_finishes():
    s = Scheduler(num_pages=20000, page_size=16, max_batch=64, max_prefill_tokens=2048, max_context=4096,
                  max_step_tokens=256)
    reqs = make(40)
    shapes, done = drive(s, reqs)
    assert len(done) == 40
    assert all(d + p <= 256 for d, p in shapes), max(d + p for d, p in shapes)
    # prompts arrive chunked: 1536 tokens over at least six steps each
    assert max(p for _, p in shapes) <= 256 and sum(p for _, p in shapes) == 40 * 1536


def test_prefill_progresses_when_decode_fills_the_cap():
    s = Scheduler(num_pages=20000, page_size=16, max_batch=64, max_prefill_tokens=2048, max_context=4096,
                  max_step_tokens=24)
    # 30 requests decode at once (> the cap of 24): each step still admits a page of prefill
    reqs = make(30, prompt=40, out=200)
    shapes, done = drive(s, reqs, arrivals_per_step=30)
    assert len(done) == 30
    assert all(d + p <= max(24, d + 16) for d, p in shapes)
    assert any(d >= 24 and p > 0 for d, p in shapes)


def test_no_cap_keeps_whole_prompt_chunks():
    s = Scheduler(num_pages=20000, page_size=16, max_batch=64, max_prefill_tokens=2048, max_context=4096)
    shapes, done = drive(s, make(5))
    assert len(done) == 5
    assert 1536 in [p for _, p in shapes]  # a whole prompt in one step


def test_summarize_steps():
    from sched_pass_b200.engine.engine import StepStats, summarize_steps
    st = [StepStats(4, 0, 4.0, True), StepStats(4, 0, 5.0, True), StepStats(4, 1536, 30.0, False)]
    s = summarize_steps(st)
    assert s["steps"] == 3 and s["decode_only_steps"] == 2 and s["mixed_or_prefill_steps"] == 1
    assert s["graph_share"] == round(2 / 3, 4) and s["decode_step_ms_p50"] == 4.0
    assert s["decode_tokens"] == 12 and s["prefill_tokens"] == 1536 and summarize_steps([]) == {"steps": 0}
    assert s["decode_tok_s_device"] == round(12 / 0.039, 1)  # 12 tokens over 39 ms of device time
