"""Continuous-batching step driver over the block pool, and the pool-churn
workload it is measured on.

s1-infer serves one sequence at a time (`generate*`, src/model/model.cpp:
252-308) and rewinds its single prefix with `truncate` (:297-298).  This
driver keeps many sequences in flight on one pool: every step it retires
finished requests (their blocks go back to the free list, or to the LRU of
the prefix cache when the cache holds them), admits queued requests while
blocks are available (longest cached prefix first shared through the
prefix cache, the rest of the prompt appended), appends one token for every
running sequence and runs decode attention for them, layer by layer, in one
batch.  No reference counterpart.

The churn workload (per GPU of a sequence-sharded box): requests arrive
Poisson-distributed, prompt lengths are log-normal, output lengths uniform,
and a fixed share of the prompts start with one of a few shared prefixes.
"""
from __future__ import annotations

import collections
import math

import numpy as np


class ChurnWorkload:
    """Seeded request stream.  Defaults are one GPU's share of an 8-GPU node
    serving 512 sequences with 8 arrivals per step: 64 running sequences,
    Poisson(1) arrivals per step; prompts log-normal (median 1024, sigma
    0.8, mean about 1410 tokens); outputs U[32, 512]; 30% of the prompts
    start with one of 16 prefixes of U[256, 4096] tokens."""

    def __init__(self, seed, arrival_rate=1.0, n_prefixes=16, prefix_len=(256, 4096), reuse=0.3,
                 prompt_median=1024, prompt_sigma=0.8, out_len=(32, 512), max_prompt=16384, vocab=1 << 20):
        self.rng = np.random.default_rng(seed)
        self.arrival_rate = arrival_rate
        self.reuse = reuse
        self.mu, self.sigma = math.log(prompt_median), prompt_sigma
        self.out_len = out_len
        self.max_prompt = max_prompt
        self.vocab = vocab
        lens = self.rng.integers(prefix_len[0], prefix_len[1] + 1, size=n_prefixes)
        self.prefixes = [self.rng.integers(0, vocab, size=int(n)).astype(np.int32) for n in lens]

    def arrivals(self):
        return int(self.rng.poisson(self.arrival_rate))

    def request(self):
        """(prompt token ids, output length).  A reusing prompt starts with
        as much of its prefix as fits."""
        n = int(min(max(round(self.rng.lognormal(self.mu, self.sigma)), 1), self.max_prompt))
        tokens = self.rng.integers(0, self.vocab, size=n).astype(np.int32)
        if self.rng.random() < self.reuse:
            pre = self.prefixes[int(self.rng.integers(len(self.prefixes)))]
            k = min(len(pre), n)
            tokens[:k] = pre[:k]
        return tokens, int(self.rng.integers(self.out_len[0], self.out_len[1] + 1))


class StepPlan:
    """One step: the sequences of the batch in order, their appended tokens
    and query rows (1 for running sequences, 0 for prompts being admitted)."""

    def __init__(self):
        self.seqs, self.n_append, self.q_lens = [], [], []
        self.admitted = []  # (seq, prompt tokens, output length)

    @property
    def n_tokens(self):
        return int(sum(self.n_append))

    @property
    def n_rows(self):
        return int(sum(self.q_lens))


class ChurnDriver:
    """Retire / admit / step bookkeeping of a continuous-batching server on
    one pool.  `pool` needs remove, prefix_match, prefix_insert, stats,
    batch(seqs, n_append, q_lens) (a context manager that reserves the
    appended tokens all-or-nothing) and block_size.  `headroom` blocks are
    kept free for the running sequences' next tokens when admitting."""

    def __init__(self, pool, workload, max_running, block_size=16, headroom=None, first_seq=1):
        self.pool, self.wl = pool, workload
        self.max_running = max_running
        self.bs = block_size
        self.headroom = max_running if headroom is None else headroom
        self.next_seq = first_seq
        self.running = collections.OrderedDict()  # seq -> remaining output tokens
        self.requests = {}  # running seq -> its request (prompt tokens, output length)
        self.queue = collections.deque()
        self.stats = collections.Counter()
        self.log = []  # bookkeeping operations in order (for replay against a reference pool)

    # ---- bookkeeping ----
    def _free_blocks(self):
        s = self.pool.stats()
        return s["num_free"] + s["num_lru"]

    def retire(self):
        done = [s for s, r in self.running.items() if r <= 0]
        for s in done:
            self.pool.remove(s)
            self.log.append(("remove", s))
            del self.running[s], self.requests[s]
        self.stats["retired"] += len(done)
        return done

    def plan(self):
        """Retires finished requests, queues arrivals, admits what fits and
        returns the step's plan (the pool is not yet touched for appends)."""
        self.retire()
        for _ in range(self.wl.arrivals()):
            self.queue.append(self.wl.request())
        plan = StepPlan()
        for s in self.running:
            plan.seqs.append(s)
            plan.n_append.append(1)
            plan.q_lens.append(1)
        avail = self._free_blocks() - self.headroom
        while self.queue and len(self.running) + len(plan.admitted) < self.max_running:
            tokens, out_len = self.queue[0]
            need = (len(tokens) + self.bs - 1) // self.bs + 1
            if need > avail:
                break
            self.queue.popleft()
            s = self.next_seq
            self.next_seq += 1
            hit = self.pool.prefix_match(s, tokens)
            self.log.append(("match", s, tokens))
            plan.seqs.append(s)
            plan.n_append.append(len(tokens) - hit)
            plan.q_lens.append(0)
            plan.admitted.append((s, tokens, out_len))
            avail -= need
            self.stats["prefix_hit_tokens"] += hit
        return plan

    def open(self, plan):
        """Opens the step's batch.  On S1KV_ENOBLOCKS (after LRU eviction)
        the admissions go back to the queue, and if the running sequences
        alone still do not fit, the longest one is preempted (its request is
        requeued from the start)."""
        from . import S1KVError, ENOBLOCKS
        while True:
            try:
                b = self.pool.batch(plan.seqs, plan.n_append, plan.q_lens)
                self.log.append(("batch", list(plan.seqs), list(plan.n_append)))
                return b
            except S1KVError as e:
                if e.status != ENOBLOCKS:
                    raise
                self.log.append(("batch_fail", list(plan.seqs), list(plan.n_append)))
            if plan.admitted:
                for s, tokens, out_len in reversed(plan.admitted):
                    self.pool.remove(s)
                    self.log.append(("remove", s))
                    self.queue.appendleft((tokens, out_len))
                n = len(plan.admitted)
                del plan.seqs[-n:], plan.n_append[-n:], plan.q_lens[-n:]
                plan.admitted = []
                self.stats["deferred"] += n
                continue
            if not plan.seqs:
                raise RuntimeError("pool too small for a single sequence")
            victim = max(plan.seqs, key=self.pool.length)
            i = plan.seqs.index(victim)
            self.pool.remove(victim)
            self.log.append(("remove", victim))
            self.queue.appendleft(self.requests.pop(victim))
            del self.running[victim], plan.seqs[i], plan.n_append[i], plan.q_lens[i]
            self.stats["preempted"] += 1

    def close(self, plan):
        """After the step's device work is enqueued: admitted prompts enter
        the prefix cache and start decoding; running sequences advance."""
        for s in plan.seqs:
            if s in self.running:
                self.running[s] -= 1
        for s, tokens, out_len in plan.admitted:
            self.pool.prefix_insert(s, tokens)
            self.log.append(("insert", s, tokens))
            self.running[s] = out_len
            self.requests[s] = (tokens, out_len)
        self.stats["admitted"] += len(plan.admitted)
        self.stats["decode_tokens"] += plan.n_rows
        self.stats["appended_tokens"] += plan.n_tokens
        self.stats["steps"] += 1
