"""Expert residency for the fused layer: a fixed number of expert slots in one device slab per
layer, with the device pointer table the kernels read.

The reference keeps recently used experts of each MoE layer in a VRAM tier and uploads a missing
expert on demand before the layer runs (`ExpertVRAMCache`, vaayu/persist/expert_cache.py:813; the
miss-upload path, vaayu/moe_patch.py:2829-2896).  `ExpertArena` is that tier for these kernels:

  * one device slab of `capacity` slots; a slot holds one expert's blob streams (packed codes,
    scales, zero points) at fixed 256-byte-aligned offsets, so any resident expert's streams are
    three addresses inside the slab;
  * `table`: the layer's pointer table [n_experts][3] for `moe_forward`, with 0 for an expert that
    is not resident (a routed expert with no streams is skipped and flagged by the kernels, never
    read);
  * `ensure(ids)`: makes every listed expert resident before a call -- a hit only refreshes its
    recency; a miss takes a free slot, or evicts the least recently used expert that the same
    call does not need.  The upload is one host-to-device copy per expert from pinned memory
    (`loader(e)` supplies the expert's blob, e.g. read from a checkpoint with
    `vaayu_b200.checkpoint`), followed by one copy of the changed table entries; both are
    enqueued on the current stream, so kernels launched after `ensure` on that stream see the new
    experts, and a slot is overwritten only after the kernels queued before it on that stream have
    read it.  Callers that launch on other streams order them against this one.

Results are bit-identical to an `ExpertTable` over the same blobs: the kernels read the same
bytes through different addresses.
"""
from __future__ import annotations

import collections
from typing import Callable, Iterable, Optional

import torch

from .moe_patch import blob_layout

_ALIGN = 256


def _round_up(n: int, a: int = _ALIGN) -> int:
    return -(-n // a) * a


class ExpertArena:
    """A layer's resident experts in one slab.  `geom`, `scale_dtype`, `has_zero`: the format every
    expert of the layer shares (a `build_expert_blob` geometry).  `loader(e)` returns expert e's
    blob (any device; CPU blobs are staged through pinned memory)."""

    def __init__(self, geom, scale_dtype: torch.dtype, has_zero: bool, n_experts: int, capacity: int,
                 loader: Callable[[int], dict], device="cuda"):
        from .packed_expert_kernels import _geom_struct
        if capacity < 1 or n_experts < 1:
            raise ValueError(f"capacity {capacity}, n_experts {n_experts}")
        self.geom, self.scale_dtype, self.has_zero = geom, scale_dtype, has_zero
        self.n_experts, self.capacity = n_experts, min(capacity, n_experts)
        self.loader = loader
        self.device = torch.device(device)
        bits, gs, roles = geom
        lay = blob_layout(geom)
        self.hidden, self.inter = lay["gate"][3], lay["gate"][2]
        words = sum(r * c * bits // 32 for _n, r, c in roles)
        scales = sum(r * c // gs for _n, r, c in roles)
        zeros = sum(-(-r * bits // 32) * (c // gs) for _n, r, c in roles) if has_zero else 0
        esz = torch.empty(0, dtype=scale_dtype).element_size()
        # byte offsets of the three streams inside a slot, and each stream's element count
        self._streams = [("packed", torch.int32, 0, words)]
        off = _round_up(words * 4)
        self._streams.append(("scale", scale_dtype, off, scales))
        off = _round_up(off + scales * esz)
        if has_zero:
            self._streams.append(("zero", torch.int32, off, zeros))
            off = _round_up(off + zeros * 4)
        self.slot_bytes = off
        raw = torch.empty(self.capacity * self.slot_bytes + _ALIGN, dtype=torch.uint8, device=self.device)
        lead = -raw.data_ptr() % _ALIGN
        self.slab = raw[lead: lead + self.capacity * self.slot_bytes]
        self._host_table = torch.zeros(n_experts * 3, dtype=torch.int64)
        self.table = torch.zeros(n_experts * 3, dtype=torch.int64, device=self.device)
        self.geom_s = _geom_struct(geom, scale_dtype, has_zero)
        self._slot_of: "collections.OrderedDict[int, int]" = collections.OrderedDict()   # LRU order
        self._free = list(range(self.capacity - 1, -1, -1))
        self.stats = collections.Counter()

    # ── the ExpertTable surface moe_forward reads ────────────────────────────────────────
    @property
    def resident(self) -> list:
        """Resident expert ids, least recently used first."""
        return list(self._slot_of)

    def weight_bytes(self, experts=None) -> int:
        idx = self.resident if experts is None else experts
        return sum(1 for e in idx if e in self._slot_of) * sum(
            n * torch.empty(0, dtype=dt).element_size() for _s, dt, _o, n in self._streams)

    def stream_views(self, slot: int) -> dict:
        """The slot's streams as typed views of the slab: {"packed", "scale"[, "zero"]}."""
        base = slot * self.slot_bytes
        return {name: self.slab[base + off: base + off + n * torch.empty(0, dtype=dt).element_size()].view(dt)
                for name, dt, off, n in self._streams}

    # ── residency ────────────────────────────────────────────────────────────────────────
    def ensure(self, ids: "Iterable[int] | torch.Tensor") -> None:
        """Make every expert in `ids` (host ids; a device tensor is read back, which synchronises)
        resident; ids outside [0, n_experts) are ignored, as the kernels drop them.  Raises when
        one call needs more experts than the arena has slots."""
        if isinstance(ids, torch.Tensor):
            ids = ids.reshape(-1).tolist()
        need = sorted({int(e) for e in ids if 0 <= int(e) < self.n_experts})
        needed = set(need)
        if len(need) > self.capacity:
            raise RuntimeError(f"ExpertArena: one call routes {len(need)} experts, the arena holds {self.capacity}")
        changed = []
        for e in need:
            if e in self._slot_of:
                self._slot_of.move_to_end(e)
                self.stats["hits"] += 1
                continue
            self.stats["misses"] += 1
            if self._free:
                slot = self._free.pop()
            else:
                victim = next(v for v in self._slot_of if v not in needed)
                slot = self._slot_of.pop(victim)
                self._host_table[3 * victim: 3 * victim + 3] = 0
                changed.append(victim)
                self.stats["evictions"] += 1
            self._upload(e, slot)
            self._slot_of[e] = slot
            changed.append(e)
        if changed:
            lo, hi = 3 * min(changed), 3 * max(changed) + 3
            self._put_table(lo, hi)

    def evict(self, e: int) -> None:
        """Drop expert e (its slot becomes free; its table entry reads 0 for later calls)."""
        slot = self._slot_of.pop(int(e), None)
        if slot is None:
            return
        self._free.append(slot)
        self._host_table[3 * e: 3 * e + 3] = 0
        self._put_table(3 * e, 3 * e + 3)
        self.stats["evictions"] += 1

    def _pinned(self, n: int) -> torch.Tensor:
        return torch.empty(n, dtype=torch.uint8, pin_memory=self.device.type == "cuda")

    def _put_table(self, lo: int, hi: int) -> None:
        """Copy host table entries [lo, hi) to the device table (one copy, current stream)."""
        host = self._pinned((hi - lo) * 8).view(torch.int64)
        host.copy_(self._host_table[lo:hi])
        self.table[lo:hi].copy_(host, non_blocking=True)

    def _upload(self, e: int, slot: int) -> None:
        blob = self.loader(e)
        if blob is None or blob["geom"] != self.geom or ("zero" in blob["flat"]) != self.has_zero \
                or blob["flat"]["scale"].dtype != self.scale_dtype:
            raise NotImplementedError(f"ExpertArena: expert {e} is not a pack-quantized blob of the layer's format")
        # one host-to-device copy of the whole slot: the streams laid out as in the slab, in a
        # pinned buffer that the caching host allocator keeps until the copy has run
        host = self._pinned(self.slot_bytes)
        for name, dt, off, n in self._streams:
            src = blob["flat"][name].reshape(-1)
            if src.numel() != n or src.dtype != dt:
                raise NotImplementedError(f"ExpertArena: expert {e}'s '{name}' stream does not match the layer")
            host[off: off + n * src.element_size()].copy_(src.detach().cpu().view(torch.uint8))
        base = slot * self.slot_bytes
        self.slab[base: base + self.slot_bytes].copy_(host, non_blocking=True)
        addr = self.slab.data_ptr() + base
        offs = {name: off for name, _dt, off, _n in self._streams}
        self._host_table[3 * e] = addr + offs["packed"]
        self._host_table[3 * e + 1] = addr + offs["scale"]
        self._host_table[3 * e + 2] = addr + offs["zero"] if self.has_zero else 0

    # ── construction from a checkpoint ───────────────────────────────────────────────────
    @classmethod
    def from_checkpoint(cls, ckpt, layer_prefix: str, capacity: int, device="cuda",
                        experts: "Optional[Iterable[int]]" = None, preload: bool = True) -> "ExpertArena":
        """An arena over the experts stored under `layer_prefix` in `ckpt` (a
        `vaayu_b200.checkpoint.Checkpoint`): expert e's blob is read from the file on its miss.
        `experts` (ascending) restricts the arena to a range -- one expert-parallel rank's share --
        whose table indexes local experts 0.. in that order; `preload` uploads the first
        `capacity` of them now."""
        ids = list(experts) if experts is not None else ckpt.experts(layer_prefix)
        if not ids:
            raise ValueError(f"no experts under {layer_prefix}")

        def loader(i: int) -> dict:
            blob = ckpt.expert_blob(layer_prefix, ids[i], device="cpu")
            if blob is None:
                raise NotImplementedError(f"{layer_prefix}.experts.{ids[i]} is not a complete pack-quantized expert")
            return blob

        first = loader(0)
        arena = cls(first["geom"], first["flat"]["scale"].dtype, "zero" in first["flat"], len(ids), capacity,
                    loader, device)
        if preload:
            arena.ensure(range(min(capacity, len(ids))))
        return arena
