"""Partial residency: a device pool of expert slots shared by several layers.

The counterpart of the reference's application-owned expert pool
(``models/flashnext/expert_pool.py:42``, ``:123-159``) and of its
slot-addressed records (``metal_runtime.py:198-228``, a route word with bit
31 set reads the pool record of that slot).  On B200 the routes stay expert
ids - the device sort needs them - and the pool carries a per-layer table
``slot_of[expert]`` on the device that the kernels read when they compute a
record's address (``vx_moe_pool.slot_of``).

A layer attached to a :class:`SlotPool` keeps its tiled records and its
routed banks in pinned host memory (the backing store, the reference's
file store); only the shared expert and the router stay on the device.  A
block call routes first, reads the routes on the host (one sync per layer, as
the reference's partial-residency path does at ``expert_cache.py:1739-1749``),
assigns slots to the routed experts (least recently used first, the
reference's ``ExpertPool.assign``), copies the misses' records from pinned
host memory into their slots on the same stream, and runs the block.  Stream
order keeps a slot from being overwritten before every earlier kernel that
read it has finished, the property the reference gets from its router sync.
"""
from __future__ import annotations

from collections import OrderedDict
from typing import Dict, Hashable, Iterable, List, Tuple

import numpy as np
import torch

from . import _lib


class SlotAssigner:
    """Host bookkeeping of (layer, expert) -> slot for `slots` slots, least
    recently used first (``expert_pool.py:123-159``): an expert already
    resident is a hit and becomes the most recent; a miss takes a free slot,
    else evicts the least recently used (layer, expert).  A request for more
    distinct experts than the pool holds fails before anything changes."""

    def __init__(self, slots: int):
        if slots < 1:
            raise ValueError("a slot pool needs at least one slot")
        self.slots = int(slots)
        self._slot_of: "OrderedDict[Tuple[Hashable, int], int]" = OrderedDict()
        self._free: List[int] = list(range(self.slots - 1, -1, -1))
        self.hits = 0
        self.misses = 0

    @property
    def usable_slots(self) -> int:
        return len(self._free) + len(self._slot_of)

    def slot(self, layer, expert: int):
        return self._slot_of.get((layer, int(expert)))

    def assign(self, layer, experts: Iterable[int]):
        """Slots for the distinct `experts` of `layer`: returns
        (slots {expert: slot}, misses [(expert, slot)] to fill, evicted
        [(layer, expert)] that lost their slot)."""
        distinct = list(dict.fromkeys(int(e) for e in experts))
        if len(distinct) > self.usable_slots:
            raise ValueError(f"{len(distinct)} experts exceed the expert pool's {self.slots} slots")
        slots: Dict[int, int] = {}
        for e in distinct:
            key = (layer, e)
            s = self._slot_of.get(key)
            if s is not None:
                self._slot_of.move_to_end(key)
                slots[e] = s
        self.hits += len(slots)
        misses, evicted = [], []
        wanted = {(layer, e) for e in distinct}
        for e in distinct:
            if e in slots:
                continue
            if self._free:
                s = self._free.pop()
            else:
                # the least recently used entry that this call does not need
                victim = next(k for k in self._slot_of if k not in wanted)
                s = self._slot_of.pop(victim)
                evicted.append(victim)
            self._slot_of[(layer, e)] = s
            slots[e] = s
            misses.append((e, s))
        self.misses += len(misses)
        return slots, misses, evicted

    def release(self, layer) -> List[Tuple[Hashable, int]]:
        """Free every slot of `layer`; returns the freed (layer, expert)."""
        gone = [k for k in self._slot_of if k[0] == layer]
        for k in gone:
            self._free.append(self._slot_of.pop(k))
        return gone


def _tile_bytes(out: int, inn: int, nproj: int, tile_rows: int, group_size: int) -> int:
    """Bytes of one expert's tiled records (``vx_q4_tiles_bytes_group`` for one expert)."""
    return int(_lib.load().vx_q4_tiles_bytes_group(1, out, inn, nproj, tile_rows, group_size))


class _Layer:
    def __init__(self, w, table: torch.Tensor, host_gu: torch.Tensor, host_dn: torch.Tensor):
        self.w = w
        self.table = table                                   # device int32 [E]
        self.mirror = np.full(table.numel(), -1, np.int32)   # host copy of the table
        self.host_gu, self.host_dn = host_gu, host_dn        # pinned records [E * stride]


class SlotPool:
    """`slots` experts' tiled records on the device, shared by the layers
    attached to it (``attach``).  Records of one slot: gate/up interleaved
    in 16-row tiles, then down in `down_rows`-row tiles, the layout of
    ``MoEWeights.pack``.  Every layer of a pool shares its quant grouping
    (`group_size` 32, or 64 for native G64 records)."""

    def __init__(self, slots: int, hidden: int, intermediate: int, down_rows: int = 32, device=None,
                 group_size: int = 32):
        if down_rows not in (16, 32):
            raise ValueError("down_rows must be 16 or 32")
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.hidden, self.intermediate, self.down_rows = int(hidden), int(intermediate), int(down_rows)
        self.group_size = int(group_size)
        self.gu_stride = _tile_bytes(self.intermediate, self.hidden, 2, 16, self.group_size)
        self.dn_stride = _tile_bytes(self.hidden, self.intermediate, 1, down_rows, self.group_size)
        if self.gu_stride == 0 or self.dn_stride == 0:
            raise ValueError(f"no tiled layout for hidden {hidden}, intermediate {intermediate}, "
                             f"group {group_size}")
        self.assigner = SlotAssigner(slots)
        self.gate_up = torch.zeros(int(slots) * self.gu_stride, dtype=torch.uint8, device=self.device)
        self.down = torch.zeros(int(slots) * self.dn_stride, dtype=torch.uint8, device=self.device)
        self._layers: Dict[int, _Layer] = {}
        self._next = 0

    @property
    def slots(self) -> int:
        return self.assigner.slots

    def attach(self, w) -> None:
        """Make `w` (a MoEWeights) a layer of this pool: its routed records
        and banks move to pinned host memory, its pool descriptor addresses
        the routed records through a device slot table (every entry -1: no
        expert resident yet).  The shared expert stays on the device."""
        if w.hidden != self.hidden or w.intermediate != self.intermediate:
            raise ValueError("layer shapes differ from the slot pool's")
        if w.group_size != self.group_size:
            raise ValueError(f"layer groups of {w.group_size} differ from the slot pool's {self.group_size}")
        if getattr(w, "slot_pool", None) is not None:
            raise ValueError("the layer is already attached to a slot pool")
        if w.pool is None or w.pool.down_rows != self.down_rows:
            w.pack(self.down_rows)
        torch.cuda.synchronize(self.device)
        host_gu = w.pool.gate_up.cpu().pin_memory()
        host_dn = w.pool.down.cpu().pin_memory()
        E = w.num_experts
        # the routed banks only give the library their shapes from here on
        for name in ("gate", "up", "down"):
            p = getattr(w, name)
            setattr(w, name, type(p)(p.weight.cpu().pin_memory(), p.scales.cpu().pin_memory(),
                                     p.biases.cpu().pin_memory(), p.group_size))
        w.pool.gate_up = self.gate_up
        w.pool.down = self.down
        table = torch.full((E,), -1, dtype=torch.int32, device=self.device)
        st = w.pool.vx()
        for name, n in (("gate_up", self.gate_up), ("down", self.down)):
            t = getattr(st, name)
            t.records = n.data_ptr()
            t.experts = self.slots
            setattr(st, name, t)
        st.slot_of = table.data_ptr()
        st.slots = self.slots
        layer = self._next
        self._next += 1
        self._layers[layer] = _Layer(w, table, host_gu, host_dn)
        w.slot_pool, w.slot_layer = self, layer

    def detach(self, w) -> None:
        """Forget `w`'s slots (its records stay in host memory; the layer
        cannot run until it is attached again)."""
        layer = w.slot_layer
        for lay, e in self.assigner.release(layer):
            self._layers[lay].mirror[e] = -1
        del self._layers[layer]
        w.slot_pool = None

    def ensure(self, w, experts: Iterable[int]) -> None:
        """Make the routed `experts` of layer `w` resident before the next
        kernel on the current stream: slots by least recent use, misses
        copied from pinned host memory, slot tables updated."""
        layer = w.slot_layer
        slots, misses, evicted = self.assigner.assign(layer, experts)
        stream = torch.cuda.current_stream(self.device)
        dirty = {layer}
        for lay, e in evicted:
            self._layers[lay].mirror[e] = -1
            dirty.add(lay)
        L = self._layers[layer]
        for e, s in misses:
            gu, dn = self.gu_stride, self.dn_stride
            self.gate_up[s * gu:(s + 1) * gu].copy_(L.host_gu[e * gu:(e + 1) * gu], non_blocking=True)
            self.down[s * dn:(s + 1) * dn].copy_(L.host_dn[e * dn:(e + 1) * dn], non_blocking=True)
        for e, s in slots.items():
            L.mirror[e] = s
        with torch.cuda.stream(stream):
            for lay in dirty:
                # a pageable source: the copy stages the table before returning,
                # so the mirror can change for the next call right away
                self._layers[lay].table.copy_(torch.from_numpy(self._layers[lay].mirror.copy()))
