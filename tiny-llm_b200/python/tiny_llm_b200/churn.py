"""Continuous-batching churn driver for the paged KV cache.

Requests arrive Poisson(rate) per step with log-uniform prompt lengths and
geometric generation lengths (seeded). Each step: admit waiting requests
while a sequence slot is free and the pool stays under its occupancy target
after taking the prompt's blocks, prefill each admitted prompt, make sure
the blocks this step's tokens need are free (otherwise release the most
recently admitted sequence and requeue it — recompute-style preemption),
run the decode step of every active sequence (one appended token per layer,
decode attention, advance), and release the sequences that reached their
generation length, returning their blocks to the free list. The cache operations are passed in, so the same
schedule drives the GPU benchmark and the CPU allocator tests.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np


@dataclass
class Request:
    prompt: int
    gen: int
    seq_id: int = -1
    generated: int = 0


@dataclass
class ChurnStats:
    steps: int = 0
    admitted: int = 0
    released: int = 0
    active_sum: int = 0
    max_active: int = 0
    tokens_attended: int = 0      # sum over steps of sum(len+1) of active sequences
    occupancy_sum: float = 0.0    # used blocks / pool blocks, summed over steps
    waiting_max: int = 0
    preempted: int = 0
    per_step_active: list = field(default_factory=list)


class ChurnSchedule:
    def __init__(self, seed=0, rate=4.0, prompt_lo=32, prompt_hi=4096, gen_mean=256,
                 max_active=256, block_size=16, occupancy_target=0.8):
        self.rng = np.random.default_rng(seed)
        self.rate, self.lo, self.hi, self.gen_mean = rate, prompt_lo, prompt_hi, gen_mean
        self.max_active, self.bs = max_active, block_size
        self.target = occupancy_target
        self.waiting: list[Request] = []
        self.active: list[Request] = []
        self.stats = ChurnStats()

    def _arrivals(self):
        n = int(self.rng.poisson(self.rate))
        out = []
        for _ in range(n):
            p = int(round(math.exp(self.rng.uniform(math.log(self.lo), math.log(self.hi)))))
            g = int(self.rng.geometric(1.0 / self.gen_mean))
            out.append(Request(prompt=max(self.lo, min(self.hi, p)), gen=max(1, g)))
        return out

    @staticmethod
    def pool_blocks_for(max_active, prompt_lo, prompt_hi, gen_mean, block_size, occupancy=0.8):
        """Pool size that keeps ~`occupancy` of the blocks in use when
        max_active sequences of mean length are resident."""
        mean_prompt = (prompt_hi - prompt_lo) / math.log(prompt_hi / prompt_lo)
        mean_len = mean_prompt + gen_mean / 2.0
        blocks = max_active * (mean_len / block_size + 0.5)
        return int(blocks / occupancy)

    def step(self, cache, prefill, decode_step, max_len):
        """One scheduler step. prefill(seq_id, prompt_len) and
        decode_step(seq_ids) perform the cache work; returns the decode
        batch (seq ids) and the attended lengths of this step."""
        self.waiting += self._arrivals()
        st = cache.pool_stats()
        free = st.free_blocks
        reserve = int((1.0 - self.target) * st.num_blocks)  # admission watermark
        while self.waiting and len(self.active) < self.max_active:
            r = self.waiting[0]
            need = -(-(r.prompt + 1) // self.bs)
            if free - need < reserve:
                break
            self.waiting.pop(0)
            r.seq_id = cache.allocate_sequence(min(max_len, r.prompt + r.gen + 1))
            prefill(r.seq_id, r.prompt)
            free -= need
            self.active.append(r)
            self.stats.admitted += 1
        # blocks this step's appended tokens start; preempt if they do not fit
        while self.active:
            need = sum(1 for r in self.active if cache.get_seq_len(r.seq_id) % self.bs == 0)
            if need <= cache.pool_stats().free_blocks:
                break
            victim = self.active.pop()
            cache.release_sequence(victim.seq_id)
            victim.seq_id, victim.generated = -1, 0
            self.waiting.insert(0, victim)
            self.stats.preempted += 1
        batch = [r.seq_id for r in self.active]
        attended = [cache.get_seq_len(s) + 1 for s in batch]
        if batch:
            decode_step(batch)
        done = []
        for r in self.active:
            r.generated += 1
            if r.generated >= r.gen or cache.get_seq_len(r.seq_id) + 1 >= min(max_len, r.prompt + r.gen + 1):
                done.append(r)
        for r in done:
            cache.release_sequence(r.seq_id)
            self.active.remove(r)
            self.stats.released += 1
        s = self.stats
        s.steps += 1
        s.active_sum += len(batch)
        s.max_active = max(s.max_active, len(batch))
        s.tokens_attended += sum(attended)
        st = cache.pool_stats()
        s.occupancy_sum += st.used_blocks / max(1, st.num_blocks)
        s.waiting_max = max(s.waiting_max, len(self.waiting))
        s.per_step_active.append(len(batch))
        return batch, attended
