"""Per-layer staging of supplier rows into local memory for the append path.

Restates ``LayerStager`` (final/cooperative_4gpu/code/peer/staging.py:6-51) as driven by the
prefill run hook (peer/prefill_backend.py:33-36 and :68-72): ``start`` once per forward after the
index list is written, ``wait(layer)`` before that layer's attention returns the local buffers that
replace the supplier banks in ``run``'s positional tail, ``next(layer)`` after the attention call
lets the buffer be refilled.

Two modes:
  * ``"range"`` (the reference's form): each bank's rows ``[begin, end)`` -- the whole bank by
    default, or the occupied range ``TierManager.remote_row_ranges`` reports -- are copied by the
    copy engines, one stream per bank (``dual_stage_bank_range``).  ``depth`` buffer sets (default
    2): layer i + depth is issued once layer i's attention is enqueued and starts when it is done,
    so with depth 2 the copy of layer i + 1 overlaps the attention of layer i with no SM work (the
    reference has one buffer per bank, so its copy of layer i + 1 follows layer i's attention).
  * ``"rows"``: only the rows the index list names are copied, by the ``stage_remote_rows`` kernel
    on the caller's stream right before the layer's attention.  For sparse use of large banks.  It
    is not overlapped: a copy CTA cannot share an SM with a running append CTA (11 warps x 160
    registers leave too few), so a concurrent copy only takes SMs from the append -- measured ~1 ms
    slower per layer than copy then append.

Why: the append kernel reads every history row once per 64-token query pair of its request and
this GPU's L2 does not cache a peer's memory, so supplier rows read in place cross NVLink many
times per layer; staged, they cross once.  Decode reads every row once, so it reads in place.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch

from . import ops
from .remote_bank import RemoteBank

LayerSource = Callable[[int], Tuple[Sequence[torch.Tensor], Sequence[torch.Tensor]]]


class LayerStager:
    def __init__(self, layer_banks: LayerSource, num_layers: int, device, depth: int = 2, mode: str = "range",
                 max_ctas: int = 0):
        """``layer_banks(i)`` gives layer i's supplier planes ``([k per bank], [v per bank])``,
        each ``[slots, 8, 128]`` bf16 (``RemoteBank.layer_kv``; see ``from_bank``).  ``max_ctas``
        bounds the ``"rows"`` kernel's grid (0 = as many CTAs as the index list needs)."""
        if mode not in ("range", "rows"):
            raise ValueError("mode must be 'range' or 'rows'")
        if depth < 1:
            raise ValueError("depth must be >= 1")
        self.layer_banks = layer_banks
        self.num_layers = int(num_layers)
        self.device = torch.device(device)
        self.mode = mode
        self.depth = depth if mode == "range" else 1
        self.max_ctas = max_ctas
        ks, vs = layer_banks(0)
        self.num_banks = len(ks)
        self.bank_slots = int(ks[0].shape[0])
        shape = tuple(ks[0].shape)
        self.buffers: List[List[Tuple[torch.Tensor, torch.Tensor]]] = [
            [(torch.empty(shape, dtype=torch.bfloat16, device=self.device),
              torch.empty(shape, dtype=torch.bfloat16, device=self.device)) for _ in ks] for _ in range(self.depth)]
        if mode == "range":
            # one copy stream per donor (staging.py:12)
            self.streams = [torch.cuda.Stream(device=self.device) for _ in ks]
            self.ready = [[torch.cuda.Event() for _ in ks] for _ in range(self.num_layers)]
            self.consumed = [torch.cuda.Event() for _ in range(self.depth)]
        self.input_ready = torch.cuda.Event()
        self.status_word = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._indices: Optional[torch.Tensor] = None
        self._count = 0
        self._capacity = 0
        self._ranges: List[Tuple[int, int]] = []
        self._launched = -1

    @classmethod
    def from_bank(cls, bank: RemoteBank, device, depth: int = 2, mode: str = "range",
                  max_ctas: int = 0) -> "LayerStager":
        return cls(bank.layer_kv, bank.layers, device, depth=depth, mode=mode, max_ctas=max_ctas)

    @property
    def bytes(self) -> int:
        """Device memory held by the stage buffers (staging.py:14-15)."""
        return sum(t.numel() * t.element_size() for s in self.buffers for pair in s for t in pair)

    def start(self, unified_indices: torch.Tensor, local_capacity: int, num_indices: Optional[int] = None,
              row_ranges: Optional[Sequence[Tuple[int, int]]] = None) -> None:
        """Begin a forward (staging.py:17-25).  ``"range"`` mode issues layers 0 .. depth-1 after the
        work already enqueued on the current stream (the packer that wrote ``unified_indices``);
        ``row_ranges`` = per bank ``(begin, end)`` rows to copy (default: the whole bank)."""
        self._indices = unified_indices
        self._count = unified_indices.numel() if num_indices is None else int(num_indices)
        self._capacity = int(local_capacity)
        if row_ranges is None:
            row_ranges = [(0, self.bank_slots)] * self.num_banks
        if len(row_ranges) != self.num_banks:
            raise ValueError("need one row range per bank")
        self._ranges = [(int(a), int(b)) for a, b in row_ranges]
        self._launched = -1
        if self.mode == "rows":
            return
        self.input_ready.record()
        for st in self.streams:
            st.wait_event(self.input_ready)
        for layer in range(min(self.depth, self.num_layers)):
            self._launch(layer)

    def _launch(self, layer: int) -> None:
        ks, vs = self.layer_banks(layer)
        buf = self.buffers[layer % self.depth]
        sk, sv = [k for k, _ in buf], [v for _, v in buf]
        if self.mode == "rows":
            ops.stage_remote_rows(ks, vs, sk, sv, self._indices, self._capacity, self.status_word,
                                  num_indices=self._count, max_ctas=self.max_ctas)
        else:
            ops.stage_bank_range(ks, vs, sk, sv, self._ranges, self.streams)
            for st, ev in zip(self.streams, self.ready[layer]):
                ev.record(st)
        self._launched = layer

    def wait(self, layer: int) -> List[Tuple[torch.Tensor, torch.Tensor]]:
        """Make the current stream wait for layer ``layer``'s rows (``"rows"``: stage them on it
        now); returns the per-bank (k, v) buffers that replace the banks in ``run``
        (staging.py:40-45)."""
        if self._indices is None:
            raise RuntimeError("call start before wait")
        if self.mode == "rows":
            self._launch(layer)
            return self.buffers[0]
        if layer > self._launched:
            raise RuntimeError(f"layer {layer} has not been staged (call next after each layer)")
        cur = torch.cuda.current_stream(self.device)
        for ev in self.ready[layer]:
            cur.wait_event(ev)
        return self.buffers[layer % self.depth]

    def tail(self, layer: int) -> List[torch.Tensor]:
        """``wait`` flattened to run's positional tail: stage_k0, stage_v0, stage_k1, ..."""
        return [t for pair in self.wait(layer) for t in pair]

    def next(self, layer: int) -> None:
        """After layer ``layer``'s attention is enqueued: refill its buffers with layer
        ``layer + depth`` once that attention is done (staging.py:47-51)."""
        if self.mode == "rows":
            return
        nxt = layer + self.depth
        if nxt >= self.num_layers:
            return
        ev = self.consumed[layer % self.depth]
        ev.record()
        for st in self.streams:
            st.wait_event(ev)
        self._launch(nxt)

    def status(self) -> int:
        """Status bits of the ``"rows"`` staging kernels so far (synchronous read)."""
        return ops.status_read(self.status_word)
