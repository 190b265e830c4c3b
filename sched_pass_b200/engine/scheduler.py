"""Continuous-batching scheduler with chunked prefill.

Every step serves all running decode requests (one token each) and fills
the remaining token budget with prefill chunks of waiting / partially
prefilled requests, oldest first. The prefill budget of a step is
``max_prefill_tokens``, further capped (when ``max_step_tokens`` > 0) so that
decode + prefill tokens stay within ``max_step_tokens``: a step whose token
count keeps every GEMM weight-bandwidth-bound costs about what a decode-only
step costs, so prefill chunks of that size ride along with the decode batch
instead of stalling it for a whole-prompt step (stall-free batching). Pages come from the native allocator; when
a decode request needs a page and none is free, the most recently admitted
request is preempted (its pages are freed and it restarts from its prompt,
keeping the tokens it already generated as part of its new prompt).
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

import numpy as np

from .native import PageAllocator
from .prefix_cache import PrefixCache
from .request import Request, State


@dataclass
class StepPlan:
    decode: list = field(default_factory=list)    # requests decoding one token
    prefill: list = field(default_factory=list)   # (request, start, n_tokens)
    preempted: list = field(default_factory=list)

    @property
    def n_tokens(self) -> int:
        return len(self.decode) + sum(n for _, _, n in self.prefill)

    @property
    def empty(self) -> bool:
        return not self.decode and not self.prefill


class Scheduler:
    def __init__(self, num_pages: int, page_size: int = 16, max_batch: int = 256,
                 max_prefill_tokens: int = 4096, max_context: int = 8192, tier=None,
                 max_step_tokens: int = 0, round_decode=None, max_prefill_segments: int = 0,
                 prefix_cache: bool = False, admission: str = "fcfs"):
        self.alloc = PageAllocator(num_pages)
        # automatic prefix caching: shared prompt prefixes reuse KV pages (engine/prefix_cache.py)
        self.cache = PrefixCache(page_size) if prefix_cache else None
        # order of admission from the waiting queue: "fcfs" (arrival), "urgency"
        # (the plane's q, highest first) or "lpm" (longest cached prefix first,
        # with the prefix cache); preempted requests always go first
        if admission not in ("fcfs", "urgency", "lpm"):
            raise ValueError(f"admission must be fcfs|urgency|lpm, not {admission!r}")
        self.admission = admission
        self.tier = tier  # optional TieredKV: spill to host before preempting
        self.page_size = page_size
        self.max_batch = max_batch
        self.max_prefill_tokens = max_prefill_tokens
        self.max_step_tokens = max_step_tokens  # 0: no cap on decode + prefill tokens
        # the engine pads decode rows to a graph bucket: the cap counts padded rows
        self.round_decode = round_decode
        self.max_prefill_segments = max_prefill_segments  # requests prefilled per step (0: any)
        self.max_context = max_context
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []   # admitted (PREFILL or DECODE), admission order
        # called before a preemption: an engine that runs ahead of the device
        # reads back pending tokens (a preempted request's output joins its prompt)
        self.before_preempt = None

    def add(self, req: Request) -> None:
        if req.prompt_len + req.max_new_tokens > self.max_context:
            raise ValueError(f"request {req.rid}: {req.prompt_len}+{req.max_new_tokens} tokens exceed "
                             f"max_context {self.max_context}")
        self.waiting.append(req)

    def admit_cached(self, req: Request, first_token: int, now: float) -> None:
        """Admit a request whose prompt K/V are already in its pages (written
        by the caller) and whose first output token is known: it joins the
        decode set directly. Used to start decode benchmarks from a warm
        cache without running their prefill."""
        if len(self.running) >= self.max_batch:
            raise RuntimeError("decode batch is full")
        if req.prompt_len + req.max_new_tokens > self.max_context:
            raise ValueError(f"request {req.rid} exceeds max_context {self.max_context}")
        if not self._grow(req, req.prompt_len):
            raise MemoryError("no free KV pages for the cached prompt")
        req.cached = req.prompt_len
        req.state = State.DECODE
        req.output.append(int(first_token))
        req.token_times.append(now)
        self.running.append(req)

    @property
    def idle(self) -> bool:
        return not self.waiting and not self.running

    @property
    def free_pages(self) -> int:
        """Pages a request can get: free ones plus cached ones nobody holds."""
        return self.alloc.free + (self.cache.evictable if self.cache is not None else 0)

    def _take(self, n: int):
        got = self.alloc.take(n)
        if got is None and self.cache is not None and self.cache.evictable:
            evicted = self.cache.evict(n - self.alloc.free)
            if evicted:
                self.alloc.give(np.asarray(evicted, dtype=np.int32))
            got = self.alloc.take(n)
        return got

    def _pages_needed(self, req: Request, upto: int) -> int:
        return max(0, (upto + self.page_size - 1) // self.page_size - len(req.pages))

    def _grow(self, req: Request, upto: int) -> bool:
        n = self._pages_needed(req, upto)
        if n == 0:
            return True
        got = self._take(n)
        if got is None and self.tier is not None:
            freed = self.tier.spill(n - self.alloc.free, self.running, protect=req)
            if freed:
                self.alloc.give(np.asarray(freed, dtype=np.int32))
            got = self.alloc.take(n)
        if got is None:
            return False
        req.pages.extend(int(p) for p in got)
        return True

    def release(self, req: Request) -> None:
        if req.pages and self.cache is not None:
            # cached pages drop this request's reference; private ones go back below
            private = []
            for p in req.pages:
                if self.cache.holds(p):
                    self.cache.release(p)
                else:
                    private.append(p)
            req.pages = private
        if req.pages:
            pages = np.asarray(req.pages, dtype=np.int64)
            if self.tier is not None:
                from .tiered_kv import HOST_BASE
                host = pages[pages >= HOST_BASE]
                if host.size:
                    self.tier.free_host(host.tolist())
                pages = pages[pages < HOST_BASE]
            self.alloc.give(pages.astype(np.int32))
            req.pages = []

    def abort(self, req: Request) -> bool:
        """Drop a request between steps, wherever it is (waiting, prefilling
        or decoding): its pages go back to the pools and it is marked DONE.
        False when the scheduler does not hold it (finished already)."""
        if req in self.running:
            self.running.remove(req)
        elif req in self.waiting:
            self.waiting.remove(req)
        else:
            return False
        self.release(req)
        req.state = State.DONE
        return True

    def _preempt(self, victim: Request, plan: StepPlan) -> None:
        if self.before_preempt is not None:
            self.before_preempt()
        self.running.remove(victim)
        self.release(victim)
        # restart from scratch: generated tokens become part of the prompt
        if victim.output:
            victim.prompt = np.concatenate([victim.prompt, np.asarray(victim.output, dtype=np.int32)])
            victim.max_new_tokens -= len(victim.output)
            victim.output = []
        victim.cached = 0
        victim.state = State.WAITING
        victim.preemptions += 1
        self.waiting.appendleft(victim)
        plan.preempted.append(victim)

    def schedule(self) -> StepPlan:
        plan = StepPlan()
        # 1. decode: every request whose prompt is fully cached
        # (a preempted request leaves `running` and becomes WAITING, so the
        # state alone says whether it is still admitted)
        for req in list(self.running):
            if req.state != State.DECODE:
                continue
            while not self._grow(req, req.total_len):
                victim = self.running[-1]
                if victim is req and len(self.running) == 1:
                    raise MemoryError("KV cache too small for a single request")
                self._preempt(victim, plan)
                if victim is req:
                    break
            if req.state == State.DECODE:
                plan.decode.append(req)
        # 2. prefill: continue partial prefills, then admit new requests
        budget = self.prefill_budget(len(plan.decode))
        seg_cap = self.max_prefill_segments or (1 << 30)
        for req in self.running:
            if budget <= 0 or len(plan.prefill) >= seg_cap:
                break
            if req.state == State.PREFILL:
                n = min(budget, req.prompt_len - req.cached)
                if n > 0 and self._grow(req, req.cached + n):
                    plan.prefill.append((req, req.cached, n))
                    budget -= n
        if self.admission != "fcfs" and len(self.waiting) > 1:
            self._order_waiting()
        while budget > 0 and self.waiting and len(self.running) < self.max_batch and len(plan.prefill) < seg_cap:
            req = self.waiting[0]
            hit_pages, keys = self.cache.peek(req.prompt, self._keys(req)) if self.cache is not None else ([], [])
            if hit_pages:
                self.cache.acquire(hit_pages)  # before growing: growing may evict idle cached pages
            req.pages = list(hit_pages)
            hit = len(hit_pages) * self.page_size
            n = min(budget, req.prompt_len - hit)
            # keep room for the decode pages of everything already running
            reserve = len(plan.decode)
            if self._pages_needed(req, hit + n) + reserve > self.free_pages or not self._grow(req, hit + n):
                if hit_pages:
                    for p in hit_pages:
                        self.cache.release(p)
                req.pages = []
                break
            if self.cache is not None:
                self.cache.lookups += req.prompt_len
                self.cache.hits += hit
            req._keys, req._registered = keys, len(hit_pages)
            req.cached = hit
            self.waiting.popleft()
            req.state = State.PREFILL
            self.running.append(req)
            plan.prefill.append((req, hit, n))
            budget -= n
        return plan

    LPM_WINDOW = 64  # waiting requests whose cached prefix is measured per step

    def _keys(self, req: Request) -> list:
        """Block keys of a request's prompt, computed once per prompt (a
        preempted request's prompt grows by its output, which renews them)."""
        memo = getattr(req, "_key_memo", None)
        if memo is None or memo[0] != req.prompt_len:
            from .prefix_cache import block_keys
            memo = (req.prompt_len, block_keys(req.prompt, self.page_size, req.prompt_len // self.page_size))
            req._key_memo = memo
        return memo[1]

    def _order_waiting(self) -> None:
        """Reorder the head of the waiting queue by the admission policy
        (stable, so ties keep arrival order; deterministic across ranks)."""
        head = [self.waiting.popleft() for _ in range(min(len(self.waiting), self.LPM_WINDOW))]
        if self.admission == "urgency":
            head.sort(key=lambda r: (r.preemptions == 0, -r.urgency))
        elif self.cache is not None:  # lpm
            head.sort(key=lambda r: (r.preemptions == 0, -len(self.cache.peek(r.prompt, self._keys(r))[0])))
        self.waiting.extendleft(reversed(head))

    def prefill_budget(self, n_decode: int) -> int:
        """Prefill tokens a step with ``n_decode`` decode tokens may add: at
        least one page's worth, so prefill always progresses."""
        if self.max_step_tokens <= 0:
            return self.max_prefill_tokens
        if self.round_decode is not None and n_decode > 0:
            n_decode = self.round_decode(n_decode)
        return min(self.max_prefill_tokens, max(self.max_step_tokens - n_decode, self.page_size))

    def commit(self, plan: StepPlan, sampled: dict, now: float) -> list:
        """Apply one step's results. ``sampled`` maps rid -> next token for
        every request that produced one. Returns the requests that finished."""
        done = []
        for req, start, n in plan.prefill:
            req.cached = start + n
            if self.cache is not None:
                # prompt blocks whose K/V this step wrote become shareable
                keys = getattr(req, "_keys", [])
                full = min(req.cached // self.page_size, len(keys))
                for b in range(getattr(req, "_registered", 0), full):
                    self.cache.register(keys[b], req.pages[b])
                req._registered = max(getattr(req, "_registered", 0), full)
            if req.cached >= req.prompt_len:
                req.state = State.DECODE
        for req in plan.decode:
            req.cached = req.total_len
        for req in list(plan.decode) + [r for r, _, _ in plan.prefill]:
            tok = sampled.get(req.rid)
            if tok is None:
                continue
            req.output.append(int(tok))
            req.token_times.append(now)
            if req.finished:
                req.state = State.DONE
                if req in self.running:
                    self.running.remove(req)
                self.release(req)
                done.append(req)
        return done
