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
     slot range per destination (T * K slots, enough for any routing; empty slots carry expert
     id -1), so the exchange needs no row counts on the host;
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

    local_blobs   the blobs of this rank's experts, in global id order
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
    """

    def __init__(self, local_blobs, n_experts: int, group=None, compute: Optional[Callable] = None,
                 combine_fn: Optional[Callable] = None, hidden: Optional[int] = None,
                 mode: str = "auto", replicate_max_tokens: int = 256,
                 layer_fn: Optional[Callable] = None, col_blocks: Optional[int] = None,
                 path: Optional[int] = None, placement: str = "contiguous"):
        if mode not in ("auto", "replicate", "dispatch"):
            raise ValueError(f"mode {mode!r}")
        if placement not in ("contiguous", "interleaved") or (placement == "interleaved" and mode != "dispatch"):
            raise ValueError(f"placement {placement!r} with mode {mode!r} (interleaved needs dispatch mode)")
        self.interleaved = placement == "interleaved"
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
            self.table = ExpertTable(local_blobs)
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

    def _dispatch_buffers(self, T, K, x, weights):
        """Fixed-capacity exchange buffers: `cap` = T * K slots per destination, enough for any
        routing (a token may even name one expert twice)."""
        key = ("dispatch", T, K, x.dtype, weights.dtype, x.device)
        b = self._bufs.get(key)
        if b is None:
            P, H, dev = self.world, x.shape[1], x.device
            cap = T * K
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
                     tok=torch.arange(T * K, device=dev) // K,
                     ranks=torch.arange(P, device=dev).view(1, P))
            self._bufs[key] = b
        return b

    def dispatch(self, x, ids, weights):
        """(recv_x, recv_local_ids, recv_w, plan) -- the rows this rank computes.  Row j of
        (token, slot) order goes to slot `dest * cap + pos` of the send buffer (pos: its rank among
        the rows for the same destination, in row order); empty slots carry expert id -1, which
        the routing plan drops.  Equal-split exchanges: no host round trip, graph-capturable."""
        T, K = ids.shape
        P = self.world
        b = self._dispatch_buffers(T, K, x, weights)
        if x.is_cuda:
            self._plan_on_device(x, ids, weights, b)
        else:
            self._plan_on_host(x, ids, weights, b)
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
                _lib.stream_of(x.device)), "vy_ep_dispatch_plan")

    def _plan_on_host(self, x, ids, weights, b):
        """The same send buffers and slot map from torch operations, for CPU tensors (the
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
        pos = hit.cumsum(0).gather(1, dest.view(-1, 1)).view(-1) - 1
        slot = dest * cap + pos
        b["slot"].copy_(slot)
        b["send_id"].fill_(-1)
        b["send_id"].index_copy_(0, slot, local.to(torch.int32))
        b["send_w"].index_copy_(0, slot, weights.reshape(-1).to(torch.float32))
        b["send_x"].index_copy_(0, slot, x.index_select(0, b["tok"]))

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
            ids_c = ids.contiguous()
            with torch.cuda.device(contrib.device):
                _lib.check(_lib.lib().vy_ep_combine(
                    b["back"].data_ptr(), slot.data_ptr(), ids_c.data_ptr(), _lib.DTYPE_CODE[ids_c.dtype], T, K,
                    self.hidden, out.data_ptr(), out.stride(0), _lib.stream_of(contrib.device)), "vy_ep_combine")
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


def run_bench(args, rank, world, local, wl):
    """bench.py's N-GPU arm: `wl` (configuration 1 or 3) at `wl['tokens']` tokens per rank (weak
    scaling), the routed experts sharded E/N per rank, steps rotating over `args.layers` layers.
    A workload with `shared` experts replicates them on every rank, applies them to the rank's own
    tokens and adds their output in bf16 (the model epilogue: out.to(bf16) + shared.to(bf16))."""
    import json
    import statistics

    import bench
    device = torch.device("cuda", local)
    E, T, K = wl["experts"], wl["tokens"], wl["top_k"]
    per = E // world
    layers = [ExpertParallelLayer(bench.make_layer(1000 * l, wl, device, (rank * per, (rank + 1) * per)), E,
                                  col_blocks=getattr(args, "ep_col_blocks", None))
              for l in range(args.layers)]
    batches = [tuple(v.to(device) for v in bench.make_tokens(l * 97 + rank, wl, T, device))
               for l in range(args.layers)]
    out = torch.empty(T, wl["hidden"], dtype=torch.float32, device=device)
    L = args.layers
    shared = None
    if wl.get("shared"):
        from .packed_expert_kernels import PATH_DECODE, ExpertTable, moe_workspace_bytes, shared_expert_forward
        sw = dict(wl, experts=1)
        shared = [ExpertTable(bench.make_layer(5000 + l, sw, device)) for l in range(L)]   # same on all ranks
        sh_out = torch.empty(T, wl["hidden"], dtype=torch.float32, device=device)
        sh_ws = torch.empty(moe_workspace_bytes(shared[0], T, 1, path=PATH_DECODE), dtype=torch.uint8, device=device)
        result = torch.empty(T, wl["hidden"], dtype=torch.bfloat16, device=device)
        if world == 1:
            # one GPU holds every expert: the shared expert rides in the same layer call as every
            # token's extra slot, the epilogue applied by the layer's combine
            from .packed_expert_kernels import _with_shared, moe_forward_with_shared
            fused_ws = torch.empty(moe_workspace_bytes(_with_shared(layers[0].table, shared[0]), T, K + 1,
                                                       path=PATH_DECODE), dtype=torch.uint8, device=device)

    def layer_step(l, x, idx, w):
        if shared is not None and world == 1:
            moe_forward_with_shared(x, idx, w, layers[l].table, shared[l], out=out, result=result,
                                    path=PATH_DECODE, workspace=fused_ws)
            return
        layers[l].forward(x, idx, w, out)
        if shared is not None:
            shared_expert_forward(x, shared[l], out=sh_out, workspace=sh_ws)
            torch.add(out.to(torch.bfloat16), sh_out.to(torch.bfloat16), out=result)

    # each layer's step (pack, all-gather, kernels, all-to-all, combine) as one CUDA graph over
    # static input buffers; eager calls when capture is not possible here
    # (each layer's inputs are views of one device record, so the end-to-end step moves them with
    # a single host-to-device copy)
    nbytes, views = bench.record_layout(batches[0])
    drecs = [torch.empty(nbytes, dtype=torch.uint8, device=device) for _ in range(L)]
    xs, ws_, ids_ = [], [], []
    for l in range(L):
        xv, wv, iv = views(drecs[l])
        for v, src in zip((xv, wv, iv), batches[l]):
            v.copy_(src)
        xs.append(xv)
        ws_.append(wv)
        ids_.append(iv)
    graphs = []
    for l in range(L):
        for _ in range(2):
            layer_step(l, xs[l], ids_[l], ws_[l])
    torch.cuda.synchronize(device)
    bench.barrier(world)
    try:
        for l in range(L):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                layer_step(l, xs[l], ids_[l], ws_[l])
            graphs.append(g)
        torch.cuda.synchronize(device)
    except Exception as e:  # noqa: BLE001 - report and run eagerly
        graphs = []
        if rank == 0:
            print(f"# EP graph capture unavailable, eager steps: {e}", flush=True)
    bench.barrier(world)

    def step(i):
        l = i % L
        if graphs:
            graphs[l].replay()
        else:
            layer_step(l, xs[l], ids_[l], ws_[l])

    for i in range(args.warmup):
        step(i)
    bench.barrier(world)
    with bench.ClockSampler(local) as clocks:
        ms = bench.time_steps(step, args.steps, device)
    bench.barrier(world)
    ms = bench.max_over_ranks(ms, world)

    pin = [bench.pinned_record(b, nbytes, views) for b in batches]
    out_h = torch.empty(T, wl["hidden"], dtype=torch.float32 if shared is None else torch.bfloat16).pin_memory()

    def e2e_step(i):
        l = i % L
        drecs[l].copy_(pin[l], non_blocking=True)
        if graphs:
            graphs[l].replay()
        else:
            layer_step(l, xs[l], ids_[l], ws_[l])
        out_h.copy_(out if shared is None else result, non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    bench.barrier(world)
    e2e_ms = bench.max_over_ranks(bench.time_steps(e2e_step, args.steps, device), world)
    bench.barrier(world)
    h2d = nbytes                      # the record copied each step (its fields padded to 16 bytes)
    used_graphs = bool(graphs)
    del graphs               # graphs holding NCCL calls go before the process group does
    torch.cuda.synchronize(device)
    uniq = statistics.mean(len(set(b[2].reshape(-1).tolist())) for b in batches)
    peak, peak_kind = bench.hbm_peak()
    if rank == 0:
        print(json.dumps({
            "metric": bench.METRIC, "value": T * world / (ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int4 weights, bf16 activations, fp32 accumulate",
            "data": "synthetic (seeded; int4 codes U{0..15}, fp16 scales U(0.005,0.02), x~N(0,1))",
            "config": {"workload": wl["name"], "hidden": wl["hidden"],
                       "expert_intermediate": wl["inter"], "experts": E, "top_k": K,
                       "tokens_per_gpu": T, "group_size": wl["group"], "layers_rotated": L,
                       "l2": "inputs larger than L2 (each layer's expert weights exceed 126 MB per step)",
                       "parallelism": f"ep{world}: {per} experts per GPU; replicate mode: one NCCL "
                                      f"all-gather of the tokens, one all-to-all of per-token partial "
                                      f"sums, rank-ordered combine",
                       "routed_experts_per_rank_batch": uniq, "cuda_graphs": used_graphs,
                       "shared_experts": wl.get("shared", 0),
                       "col_blocks": layers[0]._bufs and next(iter(layers[0]._bufs.values()))["nb"]},
            "e2e": {"value": T * world / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": out_h.numel() * out_h.element_size(),
                    "ms_per_step": e2e_ms},
            "roofline": {"kernel": "layer (expert parallel)", "bound": "hbm", "achieved": None,
                         "peak": peak, "unit": "GB/s", "frac": None, "peak_source": peak_kind,
                         "traffic": None},
            "cpu_baseline": None,
            # plan, gate/up, down and the rank-ordered sum (one GPU: the layer's combine), plus the
            # separate shared-expert call's four on several GPUs
            "gpu_launches": (4 + (4 if shared is not None and world > 1 else 0)) * args.steps,
            "clocks": clocks.summary(),
        }))


def run_prefill_bench(args, rank, world, local, wl):
    """bench.py's configuration-2 arm at any N (strong scaling): the one-GPU prefill bench's
    2048-token batches (same seeds), rank r holding tokens [r T/N, (r + 1) T/N) and experts
    r, r + N, r + 2N, ...; dispatch mode -- the rows to their experts' ranks by all-to-all (a fixed
    capacity per destination, no host round trip), the local tcgen05 prefill GEMMs, contributions
    back by the reverse all-to-all, the ascending-global-expert combine on each token's home rank.
    Each layer step is one CUDA graph."""
    import json

    import bench
    from . import synthetic
    device = torch.device("cuda", local)
    E, T, K, H, I = wl["experts"], wl["tokens"], wl["top_k"], wl["hidden"], wl["inter"]
    if E % world or T % world:
        raise ValueError(f"configuration 2 splits {E} experts and {T} tokens evenly: not over {world} GPUs")
    per, tl = E // world, T // world
    L = 2
    # round-robin placement: the benchmark's router skew grows with the expert index, which
    # contiguous ranges would hand to the last rank
    layers = [ExpertParallelLayer(bench.make_layer(2000 + l, wl, device, keep=range(rank, E, world)), E,
                                  mode="dispatch", placement="interleaved") for l in range(L)]
    batches = []
    for l in range(L):
        g = torch.Generator(device=device).manual_seed(20_000 + l)
        x, w, idx = synthetic.make_tokens(T, H, E, K, g, skew=wl["skew"])
        sl = slice(rank * tl, (rank + 1) * tl)
        batches.append((x[sl].contiguous(), w[sl].contiguous(), idx[sl].contiguous()))
    out = torch.empty(tl, H, dtype=torch.float32, device=device)
    # each layer's inputs are views of one device record (the end-to-end step fills it with one copy)
    nbytes, views = bench.record_layout(batches[0])
    drecs = [torch.empty(nbytes, dtype=torch.uint8, device=device) for _ in range(L)]
    dviews = []
    for l in range(L):
        vs = views(drecs[l])
        for v, src in zip(vs, batches[l]):
            v.copy_(src)
        dviews.append(vs)

    def layer_step(l):
        xv, wv, iv = dviews[l]
        layers[l].forward(xv, iv, wv, out)

    for l in range(L):
        for _ in range(2):
            layer_step(l)
    torch.cuda.synchronize(device)
    bench.barrier(world)
    graphs = []
    try:   # the dispatch is free of host round trips: one CUDA graph per layer step
        for l in range(L):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                layer_step(l)
            graphs.append(g)
        torch.cuda.synchronize(device)
    except Exception as e:  # noqa: BLE001 - report and run eagerly
        graphs = []
        if rank == 0:
            print(f"# EP graph capture unavailable, eager steps: {e}", flush=True)
    bench.barrier(world)

    def step(i):
        if graphs:
            graphs[i % L].replay()
        else:
            layer_step(i % L)

    for i in range(max(3, args.warmup)):
        step(i)
    steps = max(5, min(args.steps, 20))
    bench.barrier(world)
    with bench.ClockSampler(local) as clocks:
        ms = bench.time_steps(step, steps, device)
    bench.barrier(world)
    ms = bench.max_over_ranks(ms, world)

    pin = [bench.pinned_record(b, nbytes, views) for b in batches]
    out_h = torch.empty(tl, H, dtype=torch.float32).pin_memory()

    def e2e_step(i):
        l = i % L
        drecs[l].copy_(pin[l], non_blocking=True)
        step(i)
        out_h.copy_(out, non_blocking=True)

    for i in range(3):
        e2e_step(i)
    bench.barrier(world)
    e2e_ms = bench.max_over_ranks(bench.time_steps(e2e_step, steps, device), world)
    bench.barrier(world)
    used_graphs = bool(graphs)
    del graphs               # graphs holding NCCL calls go before the process group does
    torch.cuda.synchronize(device)
    flops = 2.0 * T * K * 3 * H * I
    burst, sustained, src = bench.bf16_peak()
    achieved = flops / (ms / 1e3) / 1e12 / world           # per GPU
    if rank == 0:
        print(json.dumps({
            "metric": bench.METRIC, "value": T / (ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": steps, "warmup": max(3, args.warmup), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int4 weights, bf16 activations, fp32 accumulate",
            "data": "synthetic (seeded; int4 codes U{0..15}, fp16 scales U(0.005,0.02), x~N(0,1), "
                    f"router logits skewed by linspace(0, {wl['skew']}, {E}))",
            "config": {"workload": wl["name"], "hidden": H, "expert_intermediate": I, "experts": E,
                       "top_k": K, "tokens_total": T, "tokens_per_gpu": tl, "group_size": wl["group"],
                       "layers_rotated": L, "l2": "inputs larger than L2 (each layer's expert weights: ~730 MB)",
                       "parallelism": f"ep{world}: {per} experts per GPU (round-robin); dispatch mode: "
                                      f"fixed-capacity all-to-alls of rows and contributions, "
                                      f"ascending-global-expert combine",
                       "cuda_graphs": used_graphs},
            "e2e": {"value": T / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": nbytes,
                    "d2h_bytes_per_step": out_h.numel() * out_h.element_size(), "ms_per_step": e2e_ms},
            "roofline": {"kernel": "layer (expert parallel, communication included)", "bound": "tensor",
                         "achieved": achieved, "peak": burst, "unit": "TFLOP/s", "frac": achieved / burst,
                         "peak_source": f"{src} (burst), per GPU", "traffic": None},
            "cpu_baseline": None,
            # plan, gather, gate/up GEMM, down GEMM (contributions) and the home-rank combine
            "gpu_launches": 5 * steps,
            "clocks": clocks.summary(),
        }))
