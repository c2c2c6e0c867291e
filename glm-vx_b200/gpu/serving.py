"""Batched continuous decoding of many requests on the resident decoder.

The reference scheduler (glm_vx/scheduler.py:40-243) runs one model owner
thread that interleaves requests, one token of one request per model call
(scheduler.py:160-166), each call a host round trip per kernel.  Here the
owner thread drives a ResidentDecoder (gpu/decoder.py) whose B slots decode
together: every step advances every occupied slot by one token on the device
-- the next prompt token of a slot still in its prompt, the token chosen last
step otherwise -- and the host reads back B token ids (and, for sampled
requests only, their logits rows).  A request is admitted into a free slot,
whose caches are emptied first; it leaves its slot at EOS or max_tokens.

Interface kept from the reference: submit(tokens, max_tokens, temperature,
seed) -> Request with an `events` queue of {"type": "token", "token_id"} and
a final {"type": "done", "reason", ...}; cancel(req); status(); close();
BusyError when admission capacity is exhausted; the same ValueError texts.
Greedy requests take the device argmax; temperature > 0 samples on the host
from the row's logits exactly as the reference's _sample does
(scheduler.py:113-120).  The prefix cache and batched prefill of the
reference are not rebuilt (a prompt runs through the decode steps, one
token per step, which is the reference's prefill_token semantics).
"""
from collections import deque
from dataclasses import dataclass, field
import queue
import threading
import time
import uuid

import numpy as np


class BusyError(Exception):
    pass


@dataclass
class Request:
    tokens: tuple
    max_tokens: int
    temperature: float = 0.0
    seed: int = 0
    id: str = field(default_factory=lambda: 'cmpl-' + uuid.uuid4().hex)
    events: queue.Queue = field(default_factory=queue.Queue)
    cancelled: threading.Event = field(default_factory=threading.Event)
    cursor: int = 0
    generated: int = 0
    next_token: int | None = None
    created: float = field(default_factory=time.monotonic)
    first_token_at: float | None = None
    rng: object = None
    finished: bool = False
    reservation: int = 0
    slot: int = -1
    decode_seconds: float = 0.0


class BatchScheduler:
    """Continuous batching over `decoder.B` slots of a ResidentDecoder."""

    def __init__(self, decoder, *, token_budget=None, max_pending_events=64):
        if type(max_pending_events) is not int or max_pending_events < 2:
            raise ValueError('at least two pending events required')
        self.decoder = decoder
        self.config = decoder.config
        self.slots = [None] * decoder.B
        self.token_budget = int(token_budget if token_budget is not None else decoder.B * decoder.capacity)
        self.max_pending_events = max_pending_events
        self.lock = threading.Condition()
        self.pending = deque()
        self.reserved = 0
        self.count = 0
        self.closed = False
        self.steps = 0
        self.error = None
        # Every slot advances one cache row per step, occupied or not: an
        # idle slot is emptied before it would reach the cache capacity.
        self.slot_len = [0] * decoder.B
        self.thread = threading.Thread(target=self._run, name='glm-vx-b200-decoder', daemon=True)
        self.thread.start()

    # ---------------------------------------------------------- admission
    def submit(self, tokens, max_tokens, temperature=0.0, seed=0):
        cfg = self.config
        if not isinstance(tokens, list) or not tokens or any(type(t) is not int or not 0 <= t < cfg['vocab_size']
                                                             for t in tokens):
            raise ValueError('prompt must be a nonempty array of valid token IDs')
        if type(max_tokens) is not int or max_tokens < 1:
            raise ValueError('max_tokens must be a positive integer')
        if not isinstance(temperature, (int, float)) or isinstance(temperature, bool) or \
                not np.isfinite(temperature) or temperature < 0:
            raise ValueError('temperature must be finite and nonnegative')
        if type(seed) is not int or seed < 0:
            raise ValueError('seed must be a nonnegative integer')
        amount = len(tokens) + max_tokens
        if amount > min(cfg.get('max_position_embeddings', 2**31 - 1), self.decoder.capacity):
            raise ValueError('request exceeds context limit')
        req = Request(tuple(tokens), max_tokens, float(temperature), seed)
        req.reservation = amount
        req.rng = np.random.default_rng(seed)
        req.events = queue.Queue(maxsize=min(max_tokens + 2, self.max_pending_events))
        with self.lock:
            if self.closed:
                raise BusyError('scheduler is closed')
            if self.count >= len(self.slots) or self.reserved + amount > self.token_budget:
                raise BusyError('admission capacity exhausted')
            self.reserved += amount
            self.count += 1
            self.pending.append(req)
            self.lock.notify()
        return req

    def cancel(self, req):
        req.cancelled.set()
        with self.lock:
            self.lock.notify_all()

    def status(self):
        with self.lock:
            return {'active_requests': self.count, 'reserved_tokens': self.reserved, 'slots': len(self.slots),
                    'token_budget': self.token_budget, 'max_pending_events': self.max_pending_events,
                    'steps': self.steps, 'error': self.error}

    def close(self, timeout=10):
        with self.lock:
            self.closed = True
            self.lock.notify_all()
        self.thread.join(timeout=timeout)
        if self.thread.is_alive():
            raise TimeoutError('decoder worker is still stopping')

    # -------------------------------------------------------------- worker
    def _finish(self, req, reason, error=None):
        if req.finished:
            return
        req.finished = True
        if 0 <= req.slot < len(self.slots) and self.slots[req.slot] is req:
            self.slots[req.slot] = None
        with self.lock:
            self.reserved -= req.reservation
            self.count -= 1
            self.lock.notify_all()
        try:
            req.events.put_nowait({'type': 'done', 'reason': reason, 'error': error, 'prompt_tokens': len(req.tokens),
                                   'completion_tokens': req.generated, 'cached_prompt_tokens': 0,
                                   'timings': {'prefill_seconds': 0.0, 'decode_seconds': req.decode_seconds,
                                               'prefix_seconds': 0.0}})
        except queue.Full:
            pass

    def _sample(self, logits, req):
        logits = np.asarray(logits, dtype=np.float32)
        if logits.shape != (self.config['vocab_size'],) or not np.all(np.isfinite(logits)):
            raise ValueError('nonfinite or invalid logits')
        scaled = (logits.astype(np.float64) - float(np.max(logits))) / req.temperature
        probs = np.exp(scaled)
        probs /= probs.sum()
        return int(req.rng.choice(len(probs), p=probs))

    def _admit(self):
        with self.lock:
            while not self.pending and not self.closed and not any(self.slots):
                self.lock.wait()
            arrivals = list(self.pending)
            self.pending.clear()
            closed = self.closed
        for req in arrivals:
            free = self.slots.index(None)
            req.slot = free
            self.slots[free] = req
            self.decoder.reset_slot(free)
            self.slot_len[free] = 0
        for b, r in enumerate(self.slots):
            if r is None and self.slot_len[b] >= self.decoder.capacity - 1:
                self.decoder.reset_slot(b)
                self.slot_len[b] = 0
        return closed

    def _run(self):
        dec, eos = self.decoder, self.config.get('eos_token_id', [])
        eos = [eos] if isinstance(eos, int) else list(eos or [])
        while True:
            closed = self._admit()
            for req in [r for r in self.slots if r is not None]:
                if closed or req.cancelled.is_set():
                    self._finish(req, 'cancelled')
                elif req.events.qsize() >= req.events.maxsize - 1:
                    self._finish(req, 'backpressure', 'client output queue is full')
            active = [r for r in self.slots if r is not None]
            if closed and not active:
                return
            if not active:
                continue
            try:
                feed = [0] * len(self.slots)
                for r in active:
                    feed[r.slot] = r.tokens[r.cursor] if r.cursor < len(r.tokens) else r.next_token
                t0 = time.perf_counter()
                dec.set_tokens(feed)
                dec.step()
                chosen = dec.read_tokens()
                sampled = [r for r in active if r.temperature > 0 and r.cursor + 1 >= len(r.tokens)]
                logits = dec.read_logits() if sampled else None
                dt = time.perf_counter() - t0
                self.steps += 1
                self.slot_len = [n + 1 for n in self.slot_len]
            except Exception as exc:  # the device or a bounded wait failed: every active request ends
                self.error = str(exc)
                for r in active:
                    self._finish(r, 'error', str(exc))
                continue
            for r in active:
                r.decode_seconds += dt
                if r.cursor < len(r.tokens):
                    r.cursor += 1
                    if r.cursor < len(r.tokens):
                        continue  # still inside the prompt: this step's output is not sampled
                token = self._sample(logits[r.slot], r) if r.temperature > 0 else int(chosen[r.slot])
                r.generated += 1
                r.next_token = token
                if r.first_token_at is None:
                    r.first_token_at = time.monotonic()
                r.events.put_nowait({'type': 'token', 'token_id': token})
                reason = 'stop' if token in eos else 'length' if r.generated >= r.max_tokens else None
                if reason:
                    self._finish(r, reason)


def collect(req, timeout=60.0):
    """Drain a request's events: (token ids, done event)."""
    tokens = []
    while True:
        ev = req.events.get(timeout=timeout)
        if ev['type'] == 'token':
            tokens.append(ev['token_id'])
        else:
            return tokens, ev
