"""Expert parallelism for the fused int4 expert layer: experts split across the GPUs of one node,
tokens dispatched to the ranks that hold their routed experts and combined back on the token's
home rank.

Layout: rank r holds the contiguous expert range [r * E/P, (r+1) * E/P) as a resident
`ExpertTable`; tokens start sharded (each rank owns its own batch).  One layer call:

  1. every (token, slot) row is addressed to the rank owning its expert; the per-destination row
     counts cross with one all-to-all (and come to the host: they size the variable exchange);
  2. the rows' activations, local expert ids and routing weights cross with all-to-all
     (NCCL over NVLink; peer data always lands in this GPU's own memory before a kernel reads it);
  3. each rank computes every received row's weighted contribution with the local kernels
     (`moe_forward(..., contrib=...)`, top_k = 1 per received row);
  4. the contributions (fp32) travel back with the reverse all-to-all and are put back in
     (token, slot) order;
  5. the home rank sums each token's contributions in ascending GLOBAL expert id, then slot
     (`combine`) -- `accumulate_expert_outputs`' order (vaayu/moe_patch.py:914-940).

A row's contribution does not depend on the rows it is computed with, and step 5 is the same fp32
sum in the same order as on one GPU, so the expert-parallel result equals the single-GPU result
bit for bit.  The reference is single-GPU; this module has no counterpart there.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


class ExpertParallelLayer:
    """One MoE layer's experts, sharded by contiguous ranges over the ranks of `group`.

    local_blobs   the blobs of this rank's experts, in global id order
    n_experts     the layer's total expert count (divisible by the world size)
    compute       optional (x_rows, local_ids [R,1], w_rows [R,1]) -> contributions [R, H] fp32;
                  default: the CUDA kernels over this rank's `ExpertTable`
    combine_fn    optional (contrib [T*K, H], global ids [T, K]) -> out [T, H]; default `combine`
    """

    def __init__(self, local_blobs, n_experts: int, group=None, compute: Optional[Callable] = None,
                 combine_fn: Optional[Callable] = None, hidden: Optional[int] = None):
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
        if compute is None:
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

    def dispatch(self, x, ids, weights):
        """(recv_x, recv_local_ids, recv_w, plan) -- the rows this rank computes."""
        T, K = ids.shape
        dev = x.device
        flat = ids.reshape(-1).to(torch.int64)
        dest = torch.div(flat, self.per_rank, rounding_mode="floor")
        order = torch.argsort(dest, stable=True)                 # rows grouped by destination
        send_counts = torch.bincount(dest, minlength=self.world)
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, None, None)
        sc, rc = send_counts.tolist(), recv_counts.tolist()     # host: sizes the exchange
        rows = order
        send_x = x.index_select(0, torch.div(rows, K, rounding_mode="floor"))
        send_meta = torch.stack([(flat[rows] - dest[rows] * self.per_rank).to(torch.float32),
                                 weights.reshape(-1)[rows].to(torch.float32)], dim=1)
        n_recv = int(sum(rc))
        recv_x = torch.empty(n_recv, x.shape[1], dtype=x.dtype, device=dev)
        recv_meta = torch.empty(n_recv, 2, dtype=torch.float32, device=dev)
        self._a2a(recv_x, send_x, rc, sc)
        self._a2a(recv_meta, send_meta, rc, sc)
        recv_ids = recv_meta[:, 0].to(torch.int32).view(-1, 1)
        recv_w = recv_meta[:, 1].view(-1, 1)
        if weights.dtype != torch.float32:
            # the exchange carries fp32; the routing weight keeps its own dtype for the rounding rule
            recv_w = recv_w.to(weights.dtype)
        return recv_x, recv_ids, recv_w, (order, sc, rc, T, K)

    def compute(self, recv_x, recv_ids, recv_w):
        if self._compute is not None:
            return self._compute(recv_x, recv_ids, recv_w)
        from .packed_expert_kernels import PATH_DECODE, moe_forward
        contrib = torch.empty(recv_x.shape[0], self.hidden, dtype=torch.float32, device=recv_x.device)
        if recv_x.shape[0]:
            moe_forward(recv_x, recv_ids, recv_w, self.table, contrib=contrib, path=PATH_DECODE)
        return contrib

    def gather_back(self, contrib, plan):
        order, sc, rc, T, K = plan
        back = torch.empty(T * K, contrib.shape[1], dtype=contrib.dtype, device=contrib.device)
        self._a2a(back, contrib, sc, rc)
        rows = torch.empty_like(back)
        rows[order] = back                                       # (token, slot) order again
        return rows

    def forward(self, x, ids, weights, out=None):
        """out [T, hidden] fp32 for this rank's tokens: ids are GLOBAL expert ids [T, K]."""
        recv_x, recv_ids, recv_w, plan = self.dispatch(x, ids, weights)
        contrib = self.compute(recv_x, recv_ids, recv_w)
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
    """bench.py's N-GPU arm: configuration 1 at `wl['tokens']` tokens per rank (weak scaling), the
    128 experts sharded E/N per rank, steps rotating over `args.layers` layers."""
    import json
    import statistics

    import bench
    device = torch.device("cuda", local)
    E, T, K = wl["experts"], wl["tokens"], wl["top_k"]
    per = E // world
    layers = [ExpertParallelLayer(bench.make_layer(1000 * l, wl, device, (rank * per, (rank + 1) * per)), E)
              for l in range(args.layers)]
    batches = [tuple(v.to(device) for v in bench.make_tokens(l * 97 + rank, wl, T, device))
               for l in range(args.layers)]
    out = torch.empty(T, wl["hidden"], dtype=torch.float32, device=device)
    L = args.layers

    def step(i):
        x, w, idx = batches[i % L]
        layers[i % L].forward(x, idx, w, out)

    for i in range(args.warmup):
        step(i)
    bench.barrier(world)
    with bench.ClockSampler(local) as clocks:
        ms = bench.time_steps(step, args.steps, device)
    bench.barrier(world)
    ms = bench.max_over_ranks(ms, world)

    pin = [(x.cpu().pin_memory(), w.cpu().pin_memory(), i.cpu().pin_memory()) for x, w, i in batches]
    dx, dw, di = (torch.empty_like(t) for t in batches[0])
    out_h = torch.empty(T, wl["hidden"], dtype=torch.float32).pin_memory()

    def e2e_step(i):
        xh, wh, ih = pin[i % L]
        dx.copy_(xh, non_blocking=True)
        dw.copy_(wh, non_blocking=True)
        di.copy_(ih, non_blocking=True)
        layers[i % L].forward(dx, di, dw, out)
        out_h.copy_(out, non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    bench.barrier(world)
    e2e_ms = bench.max_over_ranks(bench.time_steps(e2e_step, args.steps, device), world)
    bench.barrier(world)
    h2d = sum(t.numel() * t.element_size() for t in (dx, dw, di))
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
                       "parallelism": f"ep{world}: {per} experts per GPU, NCCL all-to-all dispatch "
                                      f"and combine", "routed_experts_per_rank_batch": uniq},
            "e2e": {"value": T * world / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": out_h.numel() * 4,
                    "ms_per_step": e2e_ms},
            "roofline": {"kernel": "layer (expert parallel)", "bound": "hbm", "achieved": None,
                         "peak": peak, "unit": "GB/s", "frac": None, "peak_source": peak_kind,
                         "traffic": None},
            "cpu_baseline": None,
            "gpu_launches": 4 * args.steps,
            "clocks": clocks.summary(),
        }))
