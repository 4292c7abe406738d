"""Expert parallelism for the fused int4 expert layer: experts split across the GPUs of one node,
tokens dispatched to the ranks that hold their routed experts and combined back on the token's
home rank.

Layout: rank r holds the contiguous expert range [r * E/P, (r+1) * E/P) as a resident
`ExpertTable`; tokens start sharded (each rank owns its own batch).  Two exchange modes:

"replicate" (decode-sized batches; no host synchronisation, two collectives):

  1. every rank's tokens -- activations, expert ids, routing weights, packed into one byte row
     per token -- are all-gathered (NCCL over NVLink);
  2. each rank runs the local kernels over all P*T tokens with only its own experts' slots kept
     (the others become -1, which the routing plan drops): per token the fp32 sum of its local
     contributions in ascending expert id (`moe_forward`'s own combine);
  3. the per-token partial sums go back to the tokens' home ranks with one equal-split
     all-to-all;
  4. the home rank adds the P partials in rank order -- ascending expert ranges.

  The result is deterministic and independent of arrival order; it groups the fp32 sum by rank
  ((sum of rank 0's slots) + (sum of rank 1's slots) + ...), so it agrees with the single-GPU
  layer to fp32 rounding, not bit for bit.

"dispatch" (large batches, where replicating every token to every rank would move too much):

  1. every (token, slot) row is addressed to the rank owning its expert, into a fixed-capacity
     slot range per destination (empty slots carry expert id -1), so the exchange needs no row
     counts on the host.  The capacity is a recorded bound, not T * K: the first call of a batch
     shape counts the rows each destination wants (one host read, all ranks agreeing on the
     largest), and later calls -- graph-capturable -- use that bound with a margin.  A call whose
     routing would overflow it drops the excess rows and raises the layer's overflow flag
     (`overflowed()`); `capacity=None` keeps T * K slots (nothing can be dropped);
  2. the rows' activations, local expert ids and routing weights cross with equal-split
     all-to-alls (NCCL over NVLink; peer data always lands in this GPU's own memory before a
     kernel reads it);
  3. each rank computes every received row's weighted contribution with the local kernels
     (`moe_forward(..., contrib=...)`, top_k = 1 per received row; the routing plan drops the
     empty slots);
  4. the contributions (fp32) travel back with the reverse all-to-all and are read out in
     (token, slot) order;
  5. the home rank sums each token's contributions in ascending GLOBAL expert id, then slot
     (`combine`) -- `accumulate_expert_outputs`' order (vaayu/moe_patch.py:914-940).

A row's contribution does not depend on the rows it is computed with, and step 5 is the same fp32
sum in the same order as on one GPU, so the dispatch-mode result equals the single-GPU result
bit for bit when both run the same kernels (`path`: the decode GEMVs or the prefill GEMMs; by
default each side picks by its own call size).  The reference is single-GPU; this module has no
counterpart there.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


class ExpertParallelLayer:
    """One MoE layer's experts, sharded by contiguous ranges over the ranks of `group`.

    local_blobs   the blobs of this rank's experts, in global id order, or a ready table of them
                  (an `ExpertTable`, or an `ExpertArena` holding every expert the rank is routed)
    n_experts     the layer's total expert count (divisible by the world size)
    mode          "replicate", "dispatch" or "auto" (replicate when every rank's batch is at most
                  `replicate_max_tokens` tokens)
    compute       optional (x_rows, local_ids [R,1], w_rows [R,1]) -> contributions [R, H] fp32;
                  dispatch mode; default: the CUDA kernels over this rank's `ExpertTable`
    combine_fn    optional (contrib [T*K, H], global ids [T, K]) -> out [T, H]; default `combine`
    layer_fn      optional (x [N, H], local ids [N, K] with -1 for other ranks' slots, w [N, K])
                  -> per-token partial sums [N, H] fp32; replicate mode; default: the CUDA kernels
    placement     "contiguous" (rank r holds [r E/P, (r+1) E/P)) or, in dispatch mode only,
                  "interleaved" (rank r holds experts r, r + P, r + 2P, ...: round-robin, which
                  spreads load that grows or shrinks with the expert index); local_blobs are the
                  rank's experts in ascending global id either way
    capacity      dispatch mode's slots per destination: "auto" (default) sizes it once per batch
                  shape from the rows the first call wants (x `capacity_margin`, agreed across
                  ranks); an int fixes it; None uses T * K (never drops a row)
    """

    def __init__(self, local_blobs, n_experts: int, group=None, compute: Optional[Callable] = None,
                 combine_fn: Optional[Callable] = None, hidden: Optional[int] = None,
                 mode: str = "auto", replicate_max_tokens: int = 256,
                 layer_fn: Optional[Callable] = None, col_blocks: Optional[int] = None,
                 path: Optional[int] = None, placement: str = "contiguous", capacity="auto",
                 capacity_margin: float = 1.5):
        if mode not in ("auto", "replicate", "dispatch"):
            raise ValueError(f"mode {mode!r}")
        if placement not in ("contiguous", "interleaved") or (placement == "interleaved" and mode != "dispatch"):
            raise ValueError(f"placement {placement!r} with mode {mode!r} (interleaved needs dispatch mode)")
        self.interleaved = placement == "interleaved"
        if not (capacity is None or capacity == "auto" or (isinstance(capacity, int) and capacity > 0)):
            raise ValueError(f"capacity {capacity!r} (\"auto\", a positive int or None)")
        self.capacity, self.capacity_margin = capacity, capacity_margin
        self._caps = {}           # (T, K) -> the recorded capacity per destination
        self._over = None         # device int32: 1 once a dispatch dropped a row
        self.mode = mode
        self.path = path      # dispatch mode's local kernels: None = moe_forward's size rule
        self.replicate_max_tokens = replicate_max_tokens
        self.col_blocks = col_blocks
        self._layer_fn = layer_fn
        self._bufs = {}
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if n_experts % self.world:
            raise ValueError(f"{n_experts} experts do not split evenly over {self.world} ranks")
        self.n_experts = n_experts
        self.per_rank = n_experts // self.world
        self.lo = self.rank * self.per_rank
        self._compute = compute
        self._combine = combine_fn
        self.table = None
        if compute is None and layer_fn is None:
            from .packed_expert_kernels import ExpertTable
            self.table = local_blobs if hasattr(local_blobs, "geom_s") else ExpertTable(local_blobs)
            self.hidden = self.table.hidden
        else:
            self.hidden = hidden

    # ── the exchange ─────────────────────────────────────────────────────────────────────
    def _a2a(self, out, inp, out_splits, in_splits):
        if self.world == 1:
            out.copy_(inp)
            return
        dist.all_to_all_single(out, inp, output_split_sizes=out_splits,
                               input_split_sizes=in_splits, group=self.group)

    def _dispatch_buffers(self, T, K, x, weights, cap=None):
        """Exchange buffers for `cap` slots per destination (default: T * K, enough for any
        routing -- a token may even name one expert twice)."""
        cap = T * K if cap is None else cap
        key = ("dispatch", T, K, cap, x.dtype, weights.dtype, x.device)
        b = self._bufs.get(key)
        if b is None:
            P, H, dev = self.world, x.shape[1], x.device
            b = dict(cap=cap,
                     send_x=torch.empty(P * cap, H, dtype=x.dtype, device=dev),
                     send_id=torch.empty(P * cap, dtype=torch.int32, device=dev),
                     send_w=torch.empty(P * cap, dtype=torch.float32, device=dev),
                     recv_x=torch.empty(P * cap, H, dtype=x.dtype, device=dev),
                     recv_id=torch.empty(P * cap, dtype=torch.int32, device=dev),
                     recv_w=torch.empty(P * cap, dtype=torch.float32, device=dev),
                     contrib=torch.empty(P * cap, H, dtype=torch.float32, device=dev),
                     back=torch.empty(P * cap, H, dtype=torch.float32, device=dev),
                     slot=torch.empty(T * K, dtype=torch.int64, device=dev),
                     counts=torch.empty(P, dtype=torch.int32, device=dev),
                     wanted=torch.empty(P, dtype=torch.int32, device=dev),
                     tok=torch.arange(T * K, device=dev) // K,
                     ranks=torch.arange(P, device=dev).view(1, P))
            self._bufs[key] = b
        return b

    def _capacity(self, T, K, x, ids, weights):
        """Slots per destination for a (T, K) batch: T * K, the fixed int, or -- "auto" -- the
        bound recorded on the first call of this shape: the rows the busiest destination wants on
        any rank, times the margin, rounded up to 8 (one host read and one MAX all-reduce; not
        inside a graph capture)."""
        if self.capacity is None:
            return T * K
        if isinstance(self.capacity, int):
            return min(self.capacity, T * K)
        cap = self._caps.get((T, K))
        if cap is None:
            probe = self._dispatch_buffers(T, K, x, weights)
            self._plan(x, ids, weights, probe)
            most = probe["wanted"].max().reshape(1).to(torch.int64)
            if self.world > 1:
                dist.all_reduce(most, op=dist.ReduceOp.MAX, group=self.group)
            cap = min(T * K, max(8, -(-int(self.capacity_margin * int(most.item())) // 8) * 8))
            self._caps[(T, K)] = cap
        return cap

    def overflowed(self) -> bool:
        """True once a dispatch call dropped a row because a destination was over its capacity
        (reads a device flag: synchronises)."""
        return bool(self._over is not None and int(self._over.item()))

    def _plan(self, x, ids, weights, b):
        if x.is_cuda:
            self._plan_on_device(x, ids, weights, b)
        else:
            self._plan_on_host(x, ids, weights, b)

    def dispatch(self, x, ids, weights):
        """(recv_x, recv_local_ids, recv_w, plan) -- the rows this rank computes.  Row j of
        (token, slot) order goes to slot `dest * cap + pos` of the send buffer (pos: its rank among
        the rows for the same destination, in row order); empty slots carry expert id -1, which
        the routing plan drops.  Equal-split exchanges: no host round trip, graph-capturable."""
        T, K = ids.shape
        b = self._dispatch_buffers(T, K, x, weights, self._capacity(T, K, x, ids, weights))
        self._plan(x, ids, weights, b)
        if b["cap"] < T * K:       # record a dropped row (no host read: graph-capturable)
            if self._over is None:
                self._over = torch.zeros(1, dtype=torch.int32, device=x.device)
            self._over.logical_or_((b["wanted"] > b["cap"]).any())
        self._a2a(b["recv_id"], b["send_id"], None, None)
        self._a2a(b["recv_w"], b["send_w"], None, None)
        self._a2a(b["recv_x"], b["send_x"], None, None)
        recv_w = b["recv_w"].view(-1, 1)
        if weights.dtype != torch.float32:
            # the exchange carries fp32; the routing weight keeps its own dtype for the rounding rule
            recv_w = recv_w.to(weights.dtype)
        return b["recv_x"], b["recv_id"].view(-1, 1), recv_w, (b["slot"], b)

    def _plan_on_device(self, x, ids, weights, b):
        """The send buffers and slot map from the library's dispatch-plan kernels (one planning
        CTA, one packing grid), on the current stream."""
        from . import _lib
        T, K = ids.shape
        weights = weights.reshape(T, K)
        if ids.stride(1) != 1:
            ids = ids.contiguous()
        if x.stride(1) != 1:
            x = x.contiguous()
        ids_code, w_code, x_code = (_lib.DTYPE_CODE[t.dtype] for t in (ids, weights, x))
        with torch.cuda.device(x.device):
            _lib.check(_lib.lib().vy_ep_dispatch_plan(
                ids.data_ptr(), ids_code, ids.stride(0), T, K, self.world, self.per_rank,
                1 if self.interleaved else 0, weights.data_ptr(), w_code, weights.stride(0), weights.stride(1),
                x.data_ptr(), x_code, x.stride(0), x.shape[1], b["cap"], b["send_id"].data_ptr(),
                b["send_w"].data_ptr(), b["send_x"].data_ptr(), b["slot"].data_ptr(), b["counts"].data_ptr(),
                b["wanted"].data_ptr(), _lib.stream_of(x.device)), "vy_ep_dispatch_plan")

    def _plan_on_host(self, x, ids, weights, b):
        """The same send buffers, slot map and counts from torch operations, for CPU tensors (the
        process-group logic's tests); every id must name one of the layer's experts."""
        T, K = ids.shape
        P, cap = self.world, b["cap"]
        flat = ids.reshape(-1).to(torch.int64)
        if self.interleaved:       # expert e lives on rank e % P as local expert e // P
            dest = torch.remainder(flat, P)
            local = torch.div(flat, P, rounding_mode="floor")
        else:
            dest = torch.div(flat, self.per_rank, rounding_mode="floor")
            local = flat - dest * self.per_rank
        # rank among the rows bound for the same destination (a running count; no host check)
        hit = (dest.view(-1, 1) == b["ranks"]).to(torch.int32)
        b["wanted"].copy_(hit.sum(0))
        b["counts"].copy_(hit.sum(0).clamp(max=cap))
        pos = hit.cumsum(0).gather(1, dest.view(-1, 1)).view(-1) - 1
        keep = pos < cap
        slot = torch.where(keep, dest * cap + pos, torch.full_like(pos, -1))
        b["slot"].copy_(slot)
        b["send_id"].fill_(-1)
        kept = keep.nonzero().view(-1)
        b["send_id"].index_copy_(0, slot[kept], local[kept].to(torch.int32))
        b["send_w"].index_copy_(0, slot[kept], weights.reshape(-1)[kept].to(torch.float32))
        b["send_x"].index_copy_(0, slot[kept], x.index_select(0, b["tok"][kept]))

    def compute(self, recv_x, recv_ids, recv_w, plan=None):
        """Contributions [P * cap, H] fp32 of the received rows (slots with id -1 stay unwritten:
        their rows are never read back)."""
        b = plan[1] if plan is not None else None
        contrib = b["contrib"] if b is not None else torch.empty(recv_x.shape[0], self.hidden, dtype=torch.float32,
                                                                    device=recv_x.device)
        if self._compute is not None:
            live = (recv_ids.view(-1) >= 0).nonzero().view(-1)    # a host-side callback sees only real rows
            if live.numel():
                contrib[live] = self._compute(recv_x[live], recv_ids[live], recv_w[live]).to(contrib.device)
            return contrib
        from .packed_expert_kernels import moe_forward
        if recv_x.shape[0]:
            moe_forward(recv_x, recv_ids, recv_w, self.table, contrib=contrib, path=self.path)
        return contrib

    def gather_back(self, contrib, plan):
        """This rank's rows' contributions back from their experts' ranks, in (token, slot) order
        (zeros for a row the dispatch dropped)."""
        slot, b = plan
        self._a2a(b["back"], contrib, None, None)
        rows = b["back"].index_select(0, slot.clamp(min=0))
        if slot.is_cuda:
            rows.masked_fill_((slot < 0).view(-1, 1), 0.0)
        return rows

    # ── replicate mode ───────────────────────────────────────────────────────────────────
    def _buffers(self, T, K, x, weights):
        key = (T, K, x.dtype, weights.dtype, x.device)
        b = self._bufs.get(key)
        if b is None:
            H = x.shape[1]
            xb, wb = 2 * H, weights.element_size() * K
            row = xb + 4 * K + wb
            row += (-row) % 16                       # 16-byte rows: the activation views stay aligned
            P = self.world
            ws = None
            # column blocks per decode pass: one unless few experts each get at most 4 rows (the
            # rank's share of the gathered slots over its experts; measured on B200, as in the
            # library's own default, which cannot see the global expert count)
            nb = self.col_blocks
            if nb is None:
                expect = T * K * P / max(1, self.n_experts)
                nb = 2 if (self.per_rank <= 16 and expect <= 4) else 1
            if self.table is not None:
                from .packed_expert_kernels import PATH_DECODE, moe_workspace_bytes
                ws = torch.empty(moe_workspace_bytes(self.table, P * T, K, path=PATH_DECODE, col_blocks=nb),
                                 dtype=torch.uint8, device=x.device)
            b = dict(row=row, xb=xb, wb=wb, ws=ws, nb=nb,
                     send=torch.empty(T, row, dtype=torch.uint8, device=x.device),
                     recv=torch.empty(P * T, row, dtype=torch.uint8, device=x.device),
                     partial=torch.empty(P * T, H, dtype=torch.float32, device=x.device),
                     back=torch.empty(P, T, H, dtype=torch.float32, device=x.device))
            self._bufs[key] = b
        return b

    def replicate_forward(self, x, ids, weights, out=None):
        """out [T, hidden] fp32: replicate mode (see the module docstring)."""
        T, K = ids.shape
        H = x.shape[1]
        P = self.world
        b = self._buffers(T, K, x, weights)
        send, recv, partial, back = b["send"], b["recv"], b["partial"], b["back"]
        xb, wb = b["xb"], b["wb"]
        send[:, :xb].view(x.dtype).copy_(x)
        send[:, xb:xb + 4 * K].view(torch.int32).copy_(ids)
        send[:, xb + 4 * K:xb + 4 * K + wb].view(weights.dtype).copy_(weights.reshape(T, K))
        if P == 1:
            recv.copy_(send)
        else:
            dist.all_gather_into_tensor(recv, send, group=self.group)
        xa = recv[:, :xb].view(x.dtype)
        ga = recv[:, xb:xb + 4 * K].view(torch.int32)
        wa = recv[:, xb + 4 * K:xb + 4 * K + wb].view(weights.dtype)
        if self._layer_fn is not None:
            local = ga - self.lo
            local = torch.where((local >= 0) & (local < self.per_rank), local, torch.full_like(local, -1))
            partial.copy_(self._layer_fn(xa, local, wa))
        else:
            # global ids straight from the gathered rows: the kernels keep [lo, lo + per_rank)
            from .packed_expert_kernels import PATH_DECODE, moe_forward
            moe_forward(xa, ga, wa, self.table, out=partial, path=PATH_DECODE, workspace=b["ws"],
                        expert_base=self.lo, col_blocks=b["nb"])
        if P == 1:
            back[0].copy_(partial)
        else:
            dist.all_to_all_single(back.view(P * T, H), partial, group=self.group)
        if out is None:
            out = torch.empty(T, H, dtype=torch.float32, device=x.device)
        if back.is_cuda and out.is_contiguous():
            from . import _lib
            with torch.cuda.device(back.device):
                # rank order: ascending expert ranges, one fp32 add each
                _lib.check(_lib.lib().vy_sum_ordered(back.data_ptr(), P, T * H, out.data_ptr(),
                                                     _lib.stream_of(back.device)), "vy_sum_ordered")
        else:
            out.copy_(back[0])
            for r in range(1, P):          # rank order: ascending expert ranges, one fp32 add each
                out.add_(back[r])
        return out

    def forward(self, x, ids, weights, out=None):
        """out [T, hidden] fp32 for this rank's tokens: ids are GLOBAL expert ids [T, K]."""
        mode = self.mode
        if mode == "auto":
            mode = "replicate" if ids.shape[0] <= self.replicate_max_tokens else "dispatch"
        if mode == "replicate":
            return self.replicate_forward(x, ids, weights, out)
        recv_x, recv_ids, recv_w, plan = self.dispatch(x, ids, weights)
        contrib = self.compute(recv_x, recv_ids, recv_w, plan)
        if self._combine is None and contrib.is_cuda:
            # the returned contributions summed in place through the slot map, ascending global
            # expert id then slot (no gathered copy)
            slot, b = plan
            self._a2a(b["back"], contrib, None, None)
            T, K = ids.shape
            if out is None:
                out = torch.empty(T, self.hidden, dtype=torch.float32, device=contrib.device)
            from . import _lib
            ids_c = ids if ids.stride(1) == 1 else ids.contiguous()
            with torch.cuda.device(contrib.device):
                _lib.check(_lib.lib().vy_ep_combine(
                    b["back"].data_ptr(), slot.data_ptr(), ids_c.data_ptr(), _lib.DTYPE_CODE[ids_c.dtype],
                    ids_c.stride(0), T, K, self.hidden, out.data_ptr(), out.stride(0),
                    _lib.stream_of(contrib.device)), "vy_ep_combine")
            return out
        rows = self.gather_back(contrib, plan)
        if self._combine is not None:
            res = self._combine(rows, ids)
            if out is not None:
                out.copy_(res)
                return out
            return res
        from .packed_expert_kernels import combine
        return combine(rows, ids, out)

