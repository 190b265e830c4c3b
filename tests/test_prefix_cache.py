"""Automatic prefix caching in the scheduler (CPU, the real allocator and
scheduler, a fake model): shared prompt prefixes are served from cached
pages, references follow the requests, idle cached pages are evicted when
the pool runs dry, every page is accounted for at every step, and two
schedulers fed the same requests make the same decisions (tensor-parallel
ranks)."""
import numpy as np

from sched_pass_b200.engine.prefix_cache import PrefixCache, block_keys
from sched_pass_b200.engine.request import Request
from sched_pass_b200.engine.scheduler import Scheduler


def step(s, now):
    plan = s.schedule()
    sampled = {r.rid: 1 for r in plan.decode}
    for r, start, n in plan.prefill:
        if start + n >= r.prompt_len:
            sampled[r.rid] = 1
    done = s.commit(plan, sampled, now)
    return plan, done


def accounted(s):
    """free + evictable + pages held by running requests (shared ones once) == pool."""
    held = set()
    for r in s.running:
        held.update(r.pages)
    cached_idle = set(s.cache.idle) if s.cache else set()
    assert not (held & cached_idle)
    return s.alloc.free + len(cached_idle) + len(held) == s.alloc.num_pages


def test_block_keys_are_prefix_chained():
    a = np.arange(64, dtype=np.int32)
    b = a.copy()
    b[40] = 7
    ka, kb = block_keys(a, 16, 4), block_keys(b, 16, 4)
    assert ka[:2] == kb[:2] and ka[2] != kb[2] and ka[3] != kb[3]


def test_shared_prefix_is_served_from_cached_pages():
    s = Scheduler(num_pages=256, page_size=16, max_batch=8, max_prefill_tokens=512, max_context=4096,
                  prefix_cache=True)
    base = np.arange(100, 164, dtype=np.int32)  # 64-token shared prefix = 4 pages
    a = Request(rid=0, prompt=np.concatenate([base, [1, 2, 3]]).astype(np.int32), max_new_tokens=20)
    s.add(a)
    plan, _ = step(s, 0.0)
    assert plan.prefill == [(a, 0, 67)]
    b = Request(rid=1, prompt=np.concatenate([base, [9, 9, 9, 9, 9]]).astype(np.int32), max_new_tokens=5)
    s.add(b)
    plan, _ = step(s, 0.1)
    assert (b, 64, 5) in plan.prefill  # only the suffix is computed
    assert b.pages[:4] == a.pages[:4] and all(s.cache.ref[p] == 2 for p in a.pages[:4])
    assert accounted(s)
    # a prompt that equals the cached prefix exactly still computes its last token
    c = Request(rid=2, prompt=base.copy(), max_new_tokens=2)
    s.add(c)
    plan, _ = step(s, 0.2)
    assert (c, 48, 16) in plan.prefill
    for t in range(40):
        step(s, 0.3 + t)
        assert accounted(s)
    assert s.idle and s.free_pages == s.alloc.num_pages
    assert s.cache.hits == 64 + 48


def test_eviction_and_accounting_under_pressure():
    rng = np.random.default_rng(0)
    prefixes = [rng.integers(0, 1000, size=int(L)).astype(np.int32) for L in (48, 96, 160)]
    s = Scheduler(num_pages=60, page_size=16, max_batch=6, max_prefill_tokens=256, max_context=1024,
                  prefix_cache=True)
    t = Scheduler(num_pages=60, page_size=16, max_batch=6, max_prefill_tokens=256, max_context=1024,
                  prefix_cache=True)
    reqs_s, reqs_t = [], []
    for i in range(60):
        p = np.concatenate([prefixes[i % 3], rng.integers(0, 1000, size=int(rng.integers(1, 40)))]).astype(np.int32)
        n_out = int(rng.integers(1, 30))
        reqs_s.append(Request(rid=i, prompt=p.copy(), max_new_tokens=n_out))
        reqs_t.append(Request(rid=i, prompt=p.copy(), max_new_tokens=n_out))
    done_s, done_t = 0, 0
    for k in range(3000):
        if k % 3 == 0 and reqs_s:
            s.add(reqs_s.pop(0))
            t.add(reqs_t.pop(0))
        if s.idle and not reqs_s:
            break
        ps, ds = step(s, float(k))
        pt, dt = step(t, float(k))
        # identical decisions on two "ranks"
        assert [(r.rid, a, n) for r, a, n in ps.prefill] == [(r.rid, a, n) for r, a, n in pt.prefill]
        assert [r.rid for r in ps.decode] == [r.rid for r in pt.decode]
        done_s += len(ds)
        done_t += len(dt)
        assert accounted(s), k
    assert done_s == done_t == 60
    assert s.cache.hits > 0 and s.free_pages == s.alloc.num_pages


def test_cache_refcounts():
    c = PrefixCache(16)
    assert c.register(b"k1", 5) and not c.register(b"k1", 6)
    c.acquire([5])
    c.release(5)
    assert c.evictable == 0
    c.release(5)
    assert c.evictable == 1 and c.evict(3) == [5] and not c.holds(5)


def test_trace_replay_prefix_reuse_becomes_cache_hits():
    """Trace records that share hash ids share token blocks (loadgen), so the
    scheduler serves the shared blocks of later requests from cached pages."""
    from sched_pass_b200.engine import loadgen

    class Fake:
        def __init__(self):
            self.sched = Scheduler(2048, 16, 8, 256, 4096, prefix_cache=True)
            self.clock = 0.0

        def add_request(self, r):
            self.sched.add(r)

        def has_work(self):
            return not self.sched.idle

        def step(self):
            plan = self.sched.schedule()
            sampled = {r.rid: 1 for r in plan.decode}
            for r, start, n in plan.prefill:
                if start + n >= r.prompt_len:
                    sampled[r.rid] = 1
            self.clock += 0.01
            return plan, self.sched.commit(plan, sampled, self.clock)

    # four conversations turns: each record extends the previous one's blocks
    recs = [{"chat_id": i, "timestamp": float(i), "input_length": 16 * (4 + 3 * i) + 5, "output_length": 2,
             "hash_ids": list(range(4 + 3 * i + 1))} for i in range(4)]
    work = loadgen.from_trace(recs, vocab=1000)
    eng = Fake()
    res, _ = loadgen.run_inprocess(eng, work)
    assert all(r.ok for r in res)
    # request i reuses the full blocks of request i-1's prompt: 4, 7, 10 blocks
    assert eng.sched.cache.hits == 16 * (4 + 7 + 10)


def test_admission_policies():
    """urgency: the most urgent waiting request is admitted first; lpm: the
    one with the longest cached prefix; fcfs keeps arrival order."""
    rng = np.random.default_rng(1)
    shared = rng.integers(0, 1000, size=96).astype(np.int32)

    def run(policy):
        s = Scheduler(num_pages=256, page_size=16, max_batch=2, max_prefill_tokens=128, max_context=4096,
                      prefix_cache=True, admission=policy)
        warm = Request(rid=0, prompt=np.concatenate([shared, [1]]).astype(np.int32), max_new_tokens=1)
        s.add(warm)
        for t in range(5):  # run the warm-up request to completion: its prefix is cached
            step(s, float(t))
        a = Request(rid=1, prompt=rng.integers(0, 1000, size=40).astype(np.int32), max_new_tokens=5, urgency=0.9)
        b = Request(rid=2, prompt=np.concatenate([shared, [2, 3]]).astype(np.int32), max_new_tokens=5,
                    urgency=0.1)
        c = Request(rid=3, prompt=rng.integers(0, 1000, size=40).astype(np.int32), max_new_tokens=5, urgency=0.5)
        for r in (c, b, a):
            s.add(r)
        plan, _ = step(s, 10.0)
        return [r.rid for r, _, _ in plan.prefill]

    assert run("fcfs")[0] == 3
    assert run("urgency")[0] == 1
    assert run("lpm")[0] == 2
