"""Token-slot migration between the local KV pool and the supplier banks.

Restates the reference's frozen 1+2+4 / 2048 policy as a standalone state
machine (no SGLang objects):

* ``budget`` / ``limit`` -- strict remote/local bound ``b*(R+m) < a*(L-m)`` in
  integers (peer/policy.py:42-46; V/nvlink_migration_latency/.../backend.py:23-25);
* ``submit`` (the reference's ``launch``, peer/policy.py:49-75) -- pins the
  oldest resident positions (FIFO, created before the previous model start),
  reserves supplier slots from ``peer_free``, runs the byte-exact copy kernel on
  a side stream ordered after the previous forward's start, records ``done``;
  the page table is NOT switched yet;
* ``poll`` -- non-blocking completion check (the reference only blocked in
  ``commit``); ``wait`` is the bounded blocking form;
* ``commit`` (peer/policy.py:78-104) -- main stream waits for ``done``, local
  sources are freed, ``tier=1`` / ``slot=target`` written, ``req_to_token`` zeroed;
* ``release`` + ``repair_active_ratio`` (V/nvlink_short_serving/.../backend.py:171-205,
  peer/policy.py:107-128) -- departing requests return their slots; if the strict
  bound breaks, the newest remote positions are restored by the reverse copy;
* ``audit`` (peer/policy.py:13-39) -- page-table invariants.

The copy itself is ``dual_b200.ops.migrate_copy`` (CUDA, one launch for all
planes); a different copier can be injected (tests drive the state machine on
the CPU with the oracle copy).
"""
from __future__ import annotations

import math
import time
from collections import Counter, deque
from dataclasses import dataclass, field
from typing import Callable, Deque, Dict, List, Optional, Sequence, Tuple

import torch

Coord = Tuple[int, int]  # (request row, logical position)


def limit_pages(local: int, remote: int, numerator: int, denominator: int) -> int:
    """Largest m with denominator*(remote+m) < numerator*(local-m) (strict, integer-exact)."""
    return max(0, (numerator * local - denominator * remote - 1) // (denominator + numerator))


class LocalAllocator:
    """Free list of local token slots 1..capacity (slot 0 is the dummy page), like SGLang's
    ``token_to_kv_pool_allocator``: ``alloc(n)`` pops n slots or returns None, ``free`` pushes back."""

    def __init__(self, capacity: int):
        self.capacity = capacity
        self._free: Deque[int] = deque(range(1, capacity + 1))

    def available_size(self) -> int:
        return len(self._free)

    def alloc(self, n: int) -> Optional[List[int]]:
        if n > len(self._free):
            return None
        return [self._free.popleft() for _ in range(n)]

    def free(self, slots: Sequence[int]) -> None:
        self._free.extend(int(s) for s in slots)


class SGLangAllocatorAdapter:
    """Drives TierManager with SGLang's own KV slot allocator (``token_to_kv_pool_allocator``:
    ``alloc(n)`` returns an index tensor or None, ``free(indices)`` takes one, ``available_size()``),
    so migrated-out local slots go back to the allocator SGLang's scheduler uses for new tokens
    (the reference frees them there too, V/nvlink_prefill_timing/backend.py:34,42)."""

    def __init__(self, allocator, device=None):
        self.inner = allocator
        self.device = device

    def available_size(self) -> int:
        return int(self.inner.available_size())

    def alloc(self, n: int) -> Optional[List[int]]:
        out = self.inner.alloc(n)
        if out is None:
            return None
        return [int(x) for x in (out.tolist() if hasattr(out, "tolist") else out)]

    def free(self, slots: Sequence[int]) -> None:
        if len(slots):
            self.inner.free(torch.tensor(list(slots), dtype=torch.int64, device=self.device))


@dataclass
class Pending:
    coords: List[Coord]
    sources: List[int]        # local slots (host mirror)
    source: torch.Tensor      # local slots (int64, device)
    target: torch.Tensor      # global remote ids (int64, device)
    targets: List[int]
    done: object              # event (torch.cuda.Event or a fake)
    record: dict = field(default_factory=dict)


class CudaCopier:
    """Production copier: the CUDA 72-plane kernel on the manager's copy stream."""

    def __init__(self, local_planes: torch.Tensor, remote_planes: torch.Tensor, num_planes: int, num_banks: int,
                 local_slots: int, remote_slots: int, status: torch.Tensor, max_ctas: int = 32):
        self.args = (local_planes, remote_planes, num_planes, num_banks)
        self.local_slots, self.remote_slots = local_slots, remote_slots
        self.status, self.max_ctas = status, max_ctas

    def __call__(self, source: torch.Tensor, target: torch.Tensor, reverse: bool) -> None:
        from . import ops
        lp, rp, planes, banks = self.args
        ops.migrate_copy(lp, rp, planes, banks, source, target, reverse, self.local_slots, self.remote_slots,
                         self.status, max_ctas=self.max_ctas)


class TierManager:
    """Local/remote page tables of one compute GPU plus the migration state machine."""

    def __init__(self, tier: torch.Tensor, slot: torch.Tensor, local_capacity: int, remote_capacity: int,
                 numerator: int, denominator: int, copier: Callable, migration_tokens: int = 2048,
                 req_to_token: Optional[torch.Tensor] = None, copy_stream=None, event_factory=None,
                 main_stream_fn=None, remote_cap: Optional[float] = None, allocator=None):
        """``remote_cap``: optional ceiling on the remote share of each request's live positions.
        The reference picks victims strictly oldest-first (``peer/policy.py:55``), which pushed its
        oldest requests to ~95 % remote; capping the share per request is the follow-up its README
        names (``README.md:128-140``).  None keeps the reference's FIFO.
        ``allocator``: the local slot allocator to draw from and free into (``LocalAllocator``
        interface, e.g. ``SGLangAllocatorAdapter`` around SGLang's); None = a private free list over
        slots 1..local_capacity."""
        if remote_cap is not None and not 0.0 < float(remote_cap) <= 1.0:
            raise ValueError("remote_cap must be in (0, 1]")
        self.remote_cap = None if remote_cap is None else float(remote_cap)
        self.tier, self.slot = tier, slot
        self.req_to_token = req_to_token
        self.local_capacity, self.remote_capacity = local_capacity, remote_capacity
        self.a, self.b = numerator, denominator
        self.copy = copier
        self.migration_tokens = migration_tokens
        self._external_allocator = allocator
        self.allocator = allocator if allocator is not None else LocalAllocator(local_capacity)
        self.device = tier.device
        cuda = self.device.type == "cuda"
        self.copy_stream = copy_stream if copy_stream is not None else (torch.cuda.Stream(self.device) if cuda else None)
        self.event_factory = event_factory or ((lambda: torch.cuda.Event()) if cuda else _HostEvent)
        self.main_stream_fn = main_stream_fn or ((lambda: torch.cuda.current_stream(self.device)) if cuda else
                                                 (lambda: None))
        self.reset()

    # ------------------------------------------------------------------ state
    def reset(self) -> None:
        self.tier.fill_(-1)
        self.slot.zero_()
        # an external allocator (SGLang's) keeps its own state; only the private free list restarts
        self.allocator = self._external_allocator or LocalAllocator(self.local_capacity)
        self.live: Dict[int, int] = {}
        self.residents: Deque[Coord] = deque()
        self.created: Dict[Coord, int] = {}
        self.peer_free: Deque[int] = deque(range(self.remote_capacity))
        self.remote_positions: Dict[Coord, int] = {}
        self.local_of: Dict[Coord, int] = {}  # host mirror of local slot ownership (no device reads)
        self.remote_counts: Counter = Counter()
        self.committed_remote = 0
        self.pending: Optional[Pending] = None
        self.step = 0
        self.model_start = None  # event recorded at the start of the latest forward
        self.migrations: List[dict] = []
        self.restorations: List[dict] = []

    def remote_row_ranges(self, num_banks: int) -> List[Tuple[int, int]]:
        """Per supplier bank, the ``[begin, end)`` physical rows that hold committed remote positions
        (host mirror, no device read; ``(0, 0)`` for a bank with none): what ``LayerStager`` copies
        in its ``"range"`` mode.  Global id ``g`` -> bank ``g % n``, row ``g // n``, the split of the
        reference's staging audit (``peer/staging.py:21-22``); the reference copies whole banks."""
        if num_banks < 1:
            raise ValueError("num_banks must be >= 1")
        lo = [None] * num_banks
        hi = [0] * num_banks
        for g in self.remote_positions.values():
            b, r = g % num_banks, g // num_banks
            lo[b] = r if lo[b] is None else min(lo[b], r)
            hi[b] = max(hi[b], r + 1)
        return [(0, 0) if lo[b] is None else (lo[b], hi[b]) for b in range(num_banks)]

    def local_active(self) -> int:
        return self.local_capacity - self.allocator.available_size()

    def budget(self) -> Tuple[int, int, int]:
        local, remote = self.local_active(), self.committed_remote
        limit = limit_pages(local, remote, self.a, self.b)
        return local, remote, min(limit, len(self.peer_free), len(self.residents))

    def amount(self, needed: int) -> Tuple[int, int, int, int]:
        local, remote, limit = self.budget()
        amount = min(self.migration_tokens, limit)
        required = max(0, needed - self.allocator.available_size())
        if amount < required:
            raise RuntimeError(f"migration budget {amount} cannot free {required} local slots "
                               f"(local={local}, remote={remote}, limit={limit})")
        return amount, local, remote, limit

    # -------------------------------------------------------------- allocation
    def begin_forward(self) -> None:
        """Mark the start of a model forward (victims must be older than this)."""
        self.step += 1
        if self.device.type == "cuda":
            ev = self.event_factory()
            ev.record(self.main_stream_fn())
            self.model_start = ev

    def append(self, rid: int, n: int) -> List[int]:
        """Allocate ``n`` new local positions at the end of request ``rid`` (prefill chunk or a decode token)."""
        start = self.live.get(rid, 0)
        slots = self.allocator.alloc(n)
        if slots is None:
            raise RuntimeError(f"local pool exhausted: need {n}, free {self.allocator.available_size()}")
        pos = list(range(start, start + n))
        idx = torch.tensor(pos, dtype=torch.long, device=self.device)
        self.slot[rid, idx] = torch.tensor(slots, dtype=torch.int32, device=self.device)
        self.tier[rid, idx] = 0
        if self.req_to_token is not None:
            self.req_to_token[rid, idx] = torch.tensor(slots, dtype=self.req_to_token.dtype, device=self.device)
        coords = [(rid, p) for p in pos]
        self.local_of.update(zip(coords, slots))
        self.residents.extend(coords)
        self.created.update((c, self.step) for c in coords)
        self.live[rid] = start + n
        return slots

    # --------------------------------------------------------------- migration
    def submit(self, needed: int = 0, asynchronous: bool = True) -> Optional[Pending]:
        """Pin victims, reserve supplier slots and launch the copy (reference ``launch``)."""
        if self.pending is not None:
            raise RuntimeError("a migration is already in flight; commit it first")
        amount, local, remote, limit = self.amount(needed)
        if amount == 0:
            return None
        selected = self._select_victims(amount, max(0, needed - self.allocator.available_size()))
        if not selected:
            return None
        amount = len(selected)
        if any(self.created[c] >= self.step for c in selected):
            # KV first written by the current forward may still be in flight.
            self.residents.extendleft(reversed(selected))
            raise RuntimeError("migration victims must predate the current forward")
        targets = [self.peer_free.popleft() for _ in selected]
        sources = [self.local_of[c] for c in selected]
        begin = time.perf_counter()
        done = self.event_factory()
        if self.device.type == "cuda" and asynchronous:
            stream = self.copy_stream
            # Victims' KV is complete once the previous forward has started (reference:
            # copy_stream.wait_event(previous model start)); do not wait for the current one.
            if self.model_start is not None:
                stream.wait_event(self.model_start)
            else:
                stream.wait_stream(self.main_stream_fn())
            with torch.cuda.stream(stream):
                source = torch.tensor(sources, dtype=torch.long, device=self.device)
                target = torch.tensor(targets, dtype=torch.long, device=self.device)
                self.copy(source, target, False)
                done.record(stream)
        else:
            source = torch.tensor(sources, dtype=torch.long, device=self.device)
            target = torch.tensor(targets, dtype=torch.long, device=self.device)
            self.copy(source, target, False)
            if self.device.type == "cuda":
                done.record(self.main_stream_fn())
            else:
                done.record()
        record = dict(tokens=amount, budget_tokens=limit, local_before=local, remote_before=remote,
                      local_after=local - amount, remote_after=remote + amount,
                      ratio_strict_pass=self.b * (remote + amount) < self.a * (local - amount),
                      copy_bytes=amount * 147456, async_copy=asynchronous, launch_step=self.step,
                      launch_cpu_ms=(time.perf_counter() - begin) * 1e3)
        if not record["ratio_strict_pass"]:
            raise AssertionError("strict remote/local bound violated by the launch")
        self.pending = Pending(selected, sources, source, target, targets, done, record)
        return self.pending

    def _select_victims(self, amount: int, required: int) -> List[Coord]:
        """Oldest resident positions first; with ``remote_cap``, positions of requests already at
        their cap are passed over (kept in place) unless the local slots that must be freed
        (``required``) cannot be found otherwise.  Positions written by the current forward are
        never eligible under a cap (FIFO raises on them, as the reference asserts)."""
        if self.remote_cap is None:
            return [self.residents.popleft() for _ in range(amount)]
        room: Dict[int, int] = {}
        chosen: List[Coord] = []
        passed: Deque[Coord] = deque()
        while self.residents and len(chosen) < amount:
            c = self.residents[0]
            if self.created[c] >= self.step:
                break  # residents are in creation order: everything after is newer still
            self.residents.popleft()
            rid = c[0]
            if rid not in room:
                room[rid] = math.floor(self.remote_cap * self.live[rid]) - self.remote_counts[rid]
            if room[rid] > 0:
                room[rid] -= 1
                chosen.append(c)
            else:
                passed.append(c)
        while len(chosen) < required and passed:  # the cap is soft when headroom must be made
            chosen.append(passed.popleft())
        chosen.sort(key=lambda k: (self.created[k], k))
        self.residents.extendleft(reversed(passed))
        return chosen

    def poll(self) -> str:
        """'idle' (nothing in flight), 'pending' (copy running) or 'ready' (commit will not wait)."""
        if self.pending is None:
            return "idle"
        return "ready" if self.pending.done.query() else "pending"

    def wait(self, timeout_s: float = 10.0) -> bool:
        """Bounded host wait for the in-flight copy; False if it did not finish in time."""
        deadline = time.monotonic() + timeout_s
        while self.poll() == "pending":
            if time.monotonic() > deadline:
                return False
            time.sleep(50e-6)
        return True

    def commit(self) -> Optional[dict]:
        """Switch the page table of the in-flight migration (reference ``commit``)."""
        if self.pending is None:
            return None
        p = self.pending
        if self.device.type == "cuda":
            self.main_stream_fn().wait_event(p.done)  # device-side ordering, no host stall
        rid = torch.tensor([r for r, _ in p.coords], dtype=torch.long, device=self.device)
        pos = torch.tensor([q for _, q in p.coords], dtype=torch.long, device=self.device)
        self.allocator.free(p.sources)
        for c in p.coords:
            del self.local_of[c]
        if self.req_to_token is not None:
            self.req_to_token[rid, pos] = 0
        self.tier[rid, pos] = 1
        self.slot[rid, pos] = torch.tensor(p.targets, dtype=torch.int32, device=self.device)
        self.committed_remote += len(p.coords)
        self.remote_positions.update(zip(p.coords, p.targets))
        self.remote_counts.update(r for r, _ in p.coords)
        local, remote, _ = self.budget()
        assert (local, remote) == (p.record["local_after"], p.record["remote_after"])
        assert self.b * remote < self.a * local
        p.record.update(commit_step=self.step)
        self.migrations.append(p.record)
        self.pending = None
        return p.record

    def ensure_headroom(self, needed: int) -> None:
        """Commit anything in flight; if local slots are still short, migrate synchronously."""
        if self.pending is not None:
            self.commit()
        if self.allocator.available_size() < needed:
            self.submit(needed, asynchronous=False)
            self.commit()

    def prefetch_next(self, batch: int) -> Optional[Pending]:
        """Start an async migration when the next step would run out of local slots."""
        if self.pending is not None or self.allocator.available_size() >= batch:
            return None
        amount = self.budget()[2]
        if amount == 0:
            return None
        oldest = list(self.residents)[: min(amount, self.migration_tokens)]
        if any(self.created[c] >= self.step for c in oldest):
            return None
        return self.submit(batch, asynchronous=True)

    # ----------------------------------------------------------------- release
    def release(self, rids: Sequence[int]) -> None:
        """Free every slot of departing requests, then restore the strict bound if it broke."""
        if self.pending is not None:
            self.commit()
        gone = set(int(r) for r in rids)
        for key in [k for k in self.remote_positions if k[0] in gone]:
            self.peer_free.append(self.remote_positions.pop(key))
            self.committed_remote -= 1
        for rid in gone:
            self.remote_counts.pop(rid, None)
        self.residents = deque(k for k in self.residents if k[0] not in gone)
        for rid in gone:
            n = self.live.pop(rid)
            near = [self.local_of.pop((rid, pos)) for pos in range(n) if (rid, pos) in self.local_of]
            for pos in range(n):
                self.created.pop((rid, pos), None)
            self.tier[rid, :n] = -1
            self.slot[rid, :n] = 0
            if self.req_to_token is not None:
                self.req_to_token[rid, :n] = 0
            self.allocator.free(near)
        self.repair_active_ratio()

    def repair_active_ratio(self) -> int:
        local, remote, _ = self.budget()
        if not remote or self.b * remote < self.a * local:
            return 0
        count = (self.b * remote - self.a * local) // (self.a + self.b) + 1
        selected = list(self.remote_positions)[-count:][::-1]  # newest remote first (reference order)
        source = torch.tensor([self.remote_positions[k] for k in selected], dtype=torch.long, device=self.device)
        slots = self.allocator.alloc(count)
        if slots is None:
            raise RuntimeError("no local slots to restore remote KV into")
        target = torch.tensor(slots, dtype=torch.long, device=self.device)
        self.copy(source, target, True)
        rid = torch.tensor([k[0] for k in selected], dtype=torch.long, device=self.device)
        pos = torch.tensor([k[1] for k in selected], dtype=torch.long, device=self.device)
        self.tier[rid, pos] = 0
        self.slot[rid, pos] = target.to(torch.int32)
        if self.req_to_token is not None:
            self.req_to_token[rid, pos] = target.to(self.req_to_token.dtype)
        for k, ls in zip(selected, slots):
            self.peer_free.append(self.remote_positions.pop(k))
            self.remote_counts[k[0]] -= 1
            self.local_of[k] = ls
        self.committed_remote -= count
        self.residents.extend(selected)
        self.residents = deque(sorted(self.residents, key=lambda k: (self.created[k], k)))
        l2, r2, _ = self.budget()
        assert not r2 or self.b * r2 < self.a * l2
        self.restorations.append(dict(tokens=count, local_before=local, remote_before=remote, local_after=l2,
                                      remote_after=r2))
        return count

    # ------------------------------------------------------------------- audit
    def audit(self) -> dict:
        """Page-table invariants of peer/policy.py:13-39 (raises AssertionError on violation)."""
        near, far, per_request = [], [], []
        for rid, n in self.live.items():
            t = self.tier[rid, :n].cpu()
            s = self.slot[rid, :n].cpu()
            f = t == 1
            assert bool(((t == 0) | f).all()), f"request {rid}: tier outside {{0, 1}}"
            if self.req_to_token is not None:
                rt = self.req_to_token[rid, :n].cpu().to(torch.int32)
                assert torch.equal(rt, torch.where(f, torch.zeros_like(s), s)), f"request {rid}: req_to_token"
            near.append(s[~f])
            far.append(s[f])
            per_request.append(dict(request=rid, context=n, local=int((~f).sum()), remote=int(f.sum())))
        n_ = torch.cat(near) if near else torch.zeros(0, dtype=torch.int32)
        f_ = torch.cat(far) if far else torch.zeros(0, dtype=torch.int32)
        reserved = len(self.pending.coords) if self.pending is not None else 0
        assert torch.unique(n_).numel() == n_.numel(), "duplicate local slots"
        assert torch.unique(f_).numel() == f_.numel(), "duplicate supplier slots"
        assert n_.numel() == self.local_active(), "local slot accounting"
        assert f_.numel() == self.committed_remote == len(self.remote_positions), "remote accounting"
        assert f_.numel() + len(self.peer_free) + reserved == self.remote_capacity, "supplier slot accounting"
        assert bool((n_ > 0).all()) and bool((n_ <= self.local_capacity).all()), "local slot range"
        assert bool((f_ >= 0).all()) and bool((f_ < self.remote_capacity).all()), "supplier slot range"
        assert not f_.numel() or self.b * f_.numel() < self.a * n_.numel(), "strict remote/local bound"
        assert +self.remote_counts == Counter(r for r, _ in self.remote_positions), "per-request remote counts"
        share = max((r["remote"] / r["context"] for r in per_request if r["context"]), default=0.0)
        return dict(local_active_tokens=int(n_.numel()), remote_active_tokens=int(f_.numel()),
                    logical_tokens=sum(self.live.values()), per_request=per_request, page_tables_exact=True,
                    max_request_remote_share=share)


class _HostEvent:
    """Event stand-in for a CPU-resident manager (copies complete synchronously)."""

    def __init__(self):
        self._done = False

    def record(self, stream=None):
        self._done = True

    def query(self) -> bool:
        return self._done

    def synchronize(self):
        pass
