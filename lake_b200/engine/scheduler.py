"""Continuous-batching step scheduler.

Each step spends a token budget: every running decode request gets one token
(decode first), then in-progress prefills and newly admitted requests get
chunks of their prompt (chunked prefill, optionally capped by
``long_prefill_threshold``). Admission reuses the longest cached prefix from
the block pool. When pages run out the most recently admitted request is
preempted and later recomputed.

Overlapped scheduling (one step in flight): advance() applies a launched step
to the host state before its tokens exist (positions advance, each sampled
request gets a PENDING token, length limits finish requests), so the next step
can be scheduled and launched while the device still runs this one; resolve()
fills the tokens in when the step completes and applies stop tokens. Before a
preemption the engine finishes the in-flight step (before_preempt), so a
preempted request never carries a PENDING token into its recomputed prompt.

Reference parity: the budget / decode-priority / chunked-extend policy of
python/lake/runtime/node_scheduler.py:396-599 (Pass A decode, Pass B extend),
the admission check against max_model_length (:96-103) and the overlap loop
with its FutureMap token relay (node_scheduler.py:190-228, future_map.py:13-30).
"""
from __future__ import annotations

import time

from collections import deque
from dataclasses import dataclass, field

from .block_pool import BlockPool, chain_block_hashes
from .request import PENDING, Request, RequestStatus


_NO_GROUP = object()  # no prefill group chosen for the step yet


@dataclass
class Chunk:
    req: Request
    start: int
    n: int
    sample: bool
    # speculative decoding: draft tokens after the request's last token; every position of
    # the chunk is sampled and `accepted` receives the verified tokens
    draft: list[int] | None = None
    accepted: list[int] | None = None

    @property
    def n_samples(self) -> int:
        if not self.sample:
            return 0
        return 1 + len(self.draft) if self.draft else 1


@dataclass
class SchedulerOutput:
    step_id: int
    decode: list[Chunk] = field(default_factory=list)
    prefill: list[Chunk] = field(default_factory=list)
    preempted: list[str] = field(default_factory=list)

    @property
    def num_tokens(self) -> int:
        return len(self.decode) + sum(c.n for c in self.prefill)

    @property
    def chunks(self) -> list[Chunk]:
        return self.decode + self.prefill

    @property
    def is_empty(self) -> bool:
        return not self.decode and not self.prefill


@dataclass
class SchedulerConfig:
    max_running: int = 256
    max_batched_tokens: int = 8192
    long_prefill_threshold: int = 0  # 0 = no per-request cap beyond the budget
    max_model_len: int = 8192
    max_blocks_per_seq: int = 512
    spec_tokens: int = 0  # draft tokens per decode request (prompt lookup); 0 = off
    spec_ngram: int = 3
    # inter-token latency target (ms) for the prefill share of mixed steps; 0 = off
    itl_target_ms: float = 0.0
    itl_min_prefill: int = 256


class ItlGovernor:
    """Prefill tokens per step, held so that the step period -- the inter-token latency every
    running decode request sees -- stays under a target.

    The period is the wall time between consecutive step completions. After a step that ran
    over the target the prefill cap shrinks by target/period (at most halving per step); after a
    step whose prefill filled the cap and ran under 90 % of the target, it grows by 10 %. The
    cap never falls below `min_tokens`, so arrivals keep being admitted, and a completion after
    an idle gap (no step in flight for over four targets) restarts the measurement. Decode rows
    are never capped: when decode alone exceeds the target, prefill runs at the floor.

    Reference parity: the ITL objective of docs/features/slo.md:15 (P50 < 50 ms), enforced by the
    node scheduler's per-step budget (python/lake/runtime/node_scheduler.py:396-430)."""

    def __init__(self, target_ms: float, max_tokens: int, min_tokens: int = 256):
        self.target = target_ms / 1000.0
        self.max = max_tokens
        self.min = min(min_tokens, max_tokens)
        self.cap = max_tokens
        self.last: float | None = None

    def observe(self, now: float, prefill_tokens: int) -> None:
        last, self.last = self.last, now
        if last is None or now - last > 4 * self.target:
            return
        period = now - last
        if period > self.target:
            self.cap = max(self.min, int(self.cap * max(0.5, self.target / period)))
        elif period < 0.9 * self.target and prefill_tokens >= 0.8 * self.cap:
            self.cap = min(self.max, int(self.cap * 1.1) + 1)

    def idle(self) -> None:
        self.last = None


class Scheduler:
    def __init__(self, pool: BlockPool, cfg: SchedulerConfig | None = None):
        self.pool = pool
        self.cfg = cfg or SchedulerConfig()
        self.bs = pool.block_size
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []
        self.step_id = 0
        self.finished: list[Request] = []
        self.on_admit = None  # callback(req) before the prefix lookup of an admission (tier promotion)
        self.before_preempt = None  # callback() before a preemption (overlap: finish the in-flight step)
        self.drafter = None
        if self.cfg.spec_tokens > 0:
            from .spec import NgramDrafter

            self.drafter = NgramDrafter(self.cfg.spec_ngram, self.cfg.spec_tokens)
        self.spec_stats = {"proposed": 0, "accepted": 0, "verify_chunks": 0}
        self.itl = (ItlGovernor(self.cfg.itl_target_ms, self.cfg.max_batched_tokens, self.cfg.itl_min_prefill)
                    if self.cfg.itl_target_ms > 0 else None)
        # group_of(req) -> key or None: prefill chunks of one step all share one key (requests
        # whose key is None join any step). A prefill instance serving several decode instances
        # keys each remote prefill by its destination, because a step's K/V stores go to one
        # destination arena. None = no constraint.
        self.group_of = None

    # -------------------------------------------------------------- admission
    def add(self, req: Request) -> None:
        if len(req.prompt) == 0:
            raise ValueError("empty prompt")
        if len(req.prompt) + req.params.max_new_tokens > self.cfg.max_model_len:
            raise ValueError(f"request {req.rid}: {len(req.prompt)}+{req.params.max_new_tokens} tokens exceed "
                             f"max_model_len {self.cfg.max_model_len}")
        req.status = RequestStatus.WAITING
        self.waiting.append(req)

    def adopt(self, req: Request) -> None:
        """Take over a request whose prompt KV is already resident in `req.block_ids`
        (prefilled by another instance); it joins the running batch in decode."""
        req.status = RequestStatus.RUNNING
        req.num_computed = len(req.prompt)
        self.running.append(req)
        self._register_full_blocks(req)

    def abort(self, rid: str) -> bool:
        for q in (self.waiting, self.running):
            for r in list(q):
                if r.rid == rid:
                    q.remove(r)
                    self._release(r)
                    r.status = RequestStatus.ABORTED
                    return True
        return False

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    # -------------------------------------------------------------- helpers
    def _blocks_needed(self, req: Request, upto: int) -> int:
        return max(0, (upto + self.bs - 1) // self.bs - len(req.block_ids))

    def _release(self, req: Request) -> None:
        if req.block_ids:
            self.pool.release(req.block_ids)
        req.block_ids = []

    def _preempt_last(self, protect: Request | None = None) -> Request | None:
        for r in reversed(self.running):
            if r is protect:
                continue
            self.running.remove(r)
            self._release(r)
            # recompute from scratch: generated tokens become part of the prompt
            r.prompt = r.prompt + r.output
            r.params.max_new_tokens -= len(r.output)
            r.meta.setdefault("preempted_output", []).extend(r.output)
            r.output = []
            r.num_computed = 0
            r.registered_blocks = 0
            r.block_hashes = []
            r.status = RequestStatus.WAITING
            self.waiting.appendleft(r)
            return r
        return None

    def _ensure_blocks(self, req: Request, upto: int, out: SchedulerOutput) -> bool:
        need = self._blocks_needed(req, upto)
        if need and not self.pool.can_alloc(need) and self.before_preempt is not None:
            self.before_preempt()  # may finish requests and free their pages
            if req.status != RequestStatus.RUNNING:
                return False
            need = self._blocks_needed(req, upto)
        while need and not self.pool.can_alloc(need):
            victim = self._preempt_last(protect=req)
            if victim is None:
                return False
            out.preempted.append(victim.rid)
            out.decode = [c for c in out.decode if c.req is not victim]
            out.prefill = [c for c in out.prefill if c.req is not victim]
        if need:
            req.block_ids += self.pool.alloc(need)
        return True

    # -------------------------------------------------------------- schedule
    def schedule(self) -> SchedulerOutput:
        out = SchedulerOutput(step_id=self.step_id)
        self.step_id += 1
        budget = self.cfg.max_batched_tokens
        # Pass A: decode
        for req in list(self.running):
            if budget <= 0:
                break
            if req.is_prefill or req.status != RequestStatus.RUNNING:
                continue
            draft = self._draft(req, budget)
            if not self._ensure_blocks(req, req.num_computed + 1 + len(draft), out):
                continue
            if req.status != RequestStatus.RUNNING:
                continue
            if draft:  # a multi-token verify chunk: runs with the prefill-shaped chunks
                out.prefill.append(Chunk(req, req.num_computed, 1 + len(draft), True, draft=draft))
                budget -= 1 + len(draft)
            else:
                out.decode.append(Chunk(req, req.num_computed, 1, True))
                budget -= 1
        # Pass B: continue chunked prefills
        cap = self.cfg.long_prefill_threshold or budget
        if self.itl is not None:  # the prefill share of a mixed step, under the latency target
            if out.decode:
                budget = min(budget, self.itl.cap)
            else:
                self.itl.idle()
        group = _NO_GROUP
        for req in list(self.running):
            if budget <= 0:
                break
            if not req.is_prefill or req.status != RequestStatus.RUNNING:
                continue
            if self.group_of is not None:
                key = self.group_of(req)
                if key is not None:
                    if group is _NO_GROUP:
                        group = key
                    elif key != group:
                        continue  # another destination: a later step
            n = min(len(req.prompt) - req.num_computed, budget, cap)
            if not self._ensure_blocks(req, req.num_computed + n, out):
                break
            out.prefill.append(Chunk(req, req.num_computed, n, req.num_computed + n == len(req.prompt)))
            budget -= n
        # Pass C: admit (with a group constraint: the oldest waiting request of the step's group,
        # or of any group when the step has none yet)
        while self.waiting and budget > 0 and len(self.running) < self.cfg.max_running:
            idx = 0
            if self.group_of is not None and group is not _NO_GROUP:
                idx = next((i for i, r in enumerate(self.waiting)
                            if self.group_of(r) is None or self.group_of(r) == group), -1)
                if idx < 0:
                    break
            req = self.waiting[idx]
            if self.group_of is not None and group is _NO_GROUP and self.group_of(req) is not None:
                group = self.group_of(req)
            if not req.block_hashes:
                req.block_hashes = chain_block_hashes(req.prompt, self.bs, full_only=True)
            usable = req.block_hashes[: (len(req.prompt) - 1) // self.bs]
            if self.on_admit is not None:
                self.on_admit(req)
            hit = self.pool.lookup(usable)
            cached = len(hit) * self.bs
            n = min(len(req.prompt) - cached, budget, cap)
            need = (cached + n + self.bs - 1) // self.bs - len(hit)
            if not self.pool.can_alloc(need):
                self.pool.release(hit)
                break
            del self.waiting[idx]
            req.block_ids = hit + self.pool.alloc(need)
            req.num_computed = cached
            req.num_cached = cached
            req.registered_blocks = len(hit)
            req.status = RequestStatus.RUNNING
            if req.admit_time is None:
                req.admit_time = time.perf_counter()
            self.running.append(req)
            out.prefill.append(Chunk(req, cached, n, cached + n == len(req.prompt)))
            budget -= n
        return out

    def _draft(self, req: Request, budget: int) -> list[int]:
        """Draft tokens for a decode request (speculative decoding), within the budget, the
        request's remaining output and the model length."""
        if self.drafter is None or req.bitmask is not None:
            return []
        room = min(budget - 1, req.params.max_new_tokens - len(req.output) - 1,
                   self.cfg.max_model_len - req.num_tokens - 1)
        if room <= 0:
            return []
        d = self.drafter.propose(req)[:room]
        if d:
            self.spec_stats["proposed"] += len(d)
            self.spec_stats["verify_chunks"] += 1
        return d

    # -------------------------------------------------------------- update
    def update(self, out: SchedulerOutput, sampled: list[int], now: float) -> list[Request]:
        """Apply one step's results. `sampled` has `n_samples` tokens per sampling chunk (one, or
        one per position of a verify chunk), in chunk order."""
        done = []
        it = iter(sampled)
        for ch in out.chunks:
            req = ch.req
            if req.status != RequestStatus.RUNNING:
                for _ in range(ch.n_samples):
                    next(it, None)
                continue
            if ch.draft:
                target = [int(next(it)) for _ in range(ch.n_samples)]
                acc = self._verify(ch.draft, target)
                self.spec_stats["accepted"] += len(acc) - 1
            else:
                req.num_computed = ch.start + ch.n
                acc = [int(next(it))] if ch.sample else []
            ch.accepted = []
            for tok in acc:
                req.output.append(tok)
                ch.accepted.append(tok)
                if req.first_token_time is None:
                    req.first_token_time = now
                req.token_times.append(now)
                if req.should_stop():
                    req.status = RequestStatus.FINISHED
                    req.finish_time = now
                    done.append(req)
                    break
            if ch.draft:  # K/V stays valid for the last token and the accepted drafts
                req.num_computed = ch.start + len(ch.accepted)
            self._register_full_blocks(req)  # after the append: accepted drafts are in its K/V
        if self.itl is not None:
            self.itl.observe(now, sum(c.n for c in out.prefill if not c.draft))
        for req in done:
            self.running.remove(req)
            self._register_full_blocks(req)
            req.meta["final_block_ids"] = list(req.block_ids)  # pages stay resident (prefix cache)
            self._release(req)
            self.finished.append(req)
        return done

    # -------------------------------------------------------------- overlapped steps
    def advance(self, out: SchedulerOutput) -> None:
        """A step was launched: advance positions, give each sampled request a PENDING token
        (meta['pslot'] = its index among the step's samples) and finish requests that reach
        their length limit (pages released now: later steps run after this one on the stream)."""
        j = 0
        for ch in out.chunks:
            req = ch.req
            slot = j
            if ch.sample:
                j += 1
            if req.status != RequestStatus.RUNNING:
                continue
            req.num_computed = ch.start + ch.n
            self._register_full_blocks(req)
            if not ch.sample:
                continue
            req.output.append(PENDING)
            req.meta["pslot"] = slot
            if len(req.output) >= req.params.max_new_tokens:
                req.status = RequestStatus.FINISHED
                req.meta["stop_pending"] = True
                self.running.remove(req)
                req.meta["final_block_ids"] = list(req.block_ids)
                self._release(req)

    def resolve(self, out: SchedulerOutput, sampled: list[int], now: float) -> list[tuple[Request, int]]:
        """The step `out` completed: replace its PENDING tokens, stamp times, apply stop tokens.
        Returns (request, token) for every token applied."""
        applied = []
        done = []
        if self.itl is not None:
            self.itl.observe(now, sum(c.n for c in out.prefill))
        it = iter(sampled)
        for ch in out.chunks:
            if not ch.sample:
                continue
            tok = int(next(it))
            req = ch.req
            if not req.output or req.output[-1] != PENDING:
                continue  # finished by a stop token one step earlier: this token is dropped
            req.output[-1] = tok
            if req.first_token_time is None:
                req.first_token_time = now
            req.token_times.append(now)
            applied.append((req, tok))
            if req.meta.pop("stop_pending", False):
                req.finish_time = now
                self.finished.append(req)
            elif req.status == RequestStatus.RUNNING and req.should_stop():
                req.status = RequestStatus.FINISHED
                req.finish_time = now
                done.append(req)
        for req in done:
            self.running.remove(req)
            req.meta["final_block_ids"] = list(req.block_ids)
            self._release(req)
            self.finished.append(req)
        return applied

    @staticmethod
    def _verify(draft: list[int], target: list[int]) -> list[int]:
        from .spec import accept

        return accept(draft, target)

    def _register_full_blocks(self, req: Request) -> None:
        full = req.num_computed // self.bs
        if full <= req.registered_blocks:
            return
        toks = req.all_tokens
        have = len(req.block_hashes)
        if have < full:
            parent = req.block_hashes[-1] if have else b""
            req.block_hashes += chain_block_hashes(toks[have * self.bs: full * self.bs], self.bs, parent=parent,
                                                   full_only=True)
        for i in range(req.registered_blocks, full):
            self.pool.register(req.block_ids[i], req.block_hashes[i])
        req.registered_blocks = full
