#!/usr/bin/env python
"""Benchmark of the fused packed-int4 MoE expert layer on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (configuration 1 of the benchmark definition, the single-GPU GEMV-bound case): a
Qwen3-30B-A3B-shaped int4 MoE layer -- hidden 2048, expert intermediate 768, 128 experts, top-8
softmax routing renormalised, int4 codes packed 8 per int32 with an fp16 scale per 128, activations
bf16 ~N(0,1) -- at a decode batch of 32 tokens (the batch 1 and 8 points are reported in
`sweep`).  A step is one layer call over one batch; steps rotate over `--layers` distinct layers
(each with its own experts and routing), so every step's ~270 MB of expert weights exceeds the
126 MB L2 and nothing is re-read from cache.  Data are seeded synthetic (no checkpoint exists here).

One JSON line on rank 0: `value` is whole-job tokens/s with inputs resident in HBM (device-timed
with CUDA events, max over ranks); `e2e` is the same metric through the public API with host
buffers (pinned H2D of x / expert ids / weights and D2H of the output inside the timed region);
`roofline` is the dominant kernel (gate/up) against the measured HBM copy bandwidth;
`cpu_baseline` is the oracle port of the reference's CPU path on this host's cores.

`--impl reference` times the reference's CPU implementation of the path -- the oracle port of
`stock_experts_prefill(linear=_linear_fp32)` (the reference is Python and cannot travel to the
GPU host) -- on the same workload, with all host threads.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "int4 MoE expert-layer tokens/s and % HBM/tensor roofline at 1/2/4/8 B200"
WORKLOAD = dict(name="cfg1: Qwen3-30B-A3B-shaped int4 MoE layer, decode", hidden=2048, inter=768,
                experts=128, top_k=8, tokens=32, group=128)
CFG3 = dict(name="cfg3: DeepSeek-V3-shaped int4 MoE layer (256 routed experts, top-8, 1 shared), "
                 "expert-parallel decode", hidden=7168, inter=2048, experts=256, top_k=8, tokens=64,
            group=128, shared=1, zeros=True)   # zero points U{0..15} per (row, group), as configuration 3 asks
PREFILL = dict(name="cfg2: Mixtral-8x7B-shaped int4 MoE layer, prefill", hidden=4096, inter=14336,
               experts=8, top_k=2, tokens=2048, group=128, skew=0.9)
CFG3_PREFILL = dict(name="cfg3: DeepSeek-V3-shaped int4 MoE layer (256 routed experts, top-8, 1 shared), "
                         "expert-parallel prefill", hidden=7168, inter=2048, experts=256, top_k=8, tokens=4096,
                    group=128, shared=1, zeros=True)
PEAKS = ROOT / "MEASURED_PEAKS.json"
FALLBACK_HBM = 6650.0
FALLBACK_BF16 = 1590.0


def hbm_peak():
    try:
        return float(json.loads(PEAKS.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM, "fallback"


def bf16_peak():
    """(burst TFLOP/s, sustained TFLOP/s or None, source)."""
    try:
        p = json.loads(PEAKS.read_text())
        return float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained") or 0) or None, "measured"
    except Exception:
        return FALLBACK_BF16, None, "fallback"


# ── distributed plumbing ─────────────────────────────────────────────────────────────────

def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ── clocks ───────────────────────────────────────────────────────────────────────────────

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out = self.proc.communicate(timeout=5)[0]
            except Exception:
                self.proc.kill()
                self.out = ""

    def summary(self):
        if self.proc is None or not getattr(self, "out", ""):
            return None
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ── workload ─────────────────────────────────────────────────────────────────────────────

def make_layer(seed, wl, device, experts_slice=None, keep=None):
    """One layer's expert blobs (generated on the device from a seeded CUDA generator): all of
    them, the range `experts_slice` = (lo, hi), or the ids in `keep`, in ascending id."""
    import vaayu_b200 as vb
    from vaayu_b200 import synthetic
    g = torch.Generator(device=device).manual_seed(seed)
    blobs = []
    lo, hi = experts_slice or (0, wl["experts"])
    keep = set(keep) if keep is not None else set(range(lo, hi))
    for e in range(wl["experts"]):
        by_role = synthetic.make_expert(wl["hidden"], wl["inter"], g, group=wl["group"], zeros=wl.get("zeros", False))
        if e in keep:
            blobs.append(vb.build_expert_blob(by_role))
    return blobs


def make_tokens(seed, wl, tokens, device):
    from vaayu_b200 import synthetic
    g = torch.Generator(device=device).manual_seed(10_000 + seed)
    return synthetic.make_tokens(tokens, wl["hidden"], wl["experts"], wl["top_k"], g)


def unique_bytes(table, idx):
    ids = sorted(set(idx.reshape(-1).tolist()))
    return table.weight_bytes(ids), len(ids)


def gate_up_bytes(table, idx):
    """Algorithmic bytes of the gate/up stage: the routed experts' gate + up codes and scales."""
    from vaayu_b200.moe_patch import blob_layout
    lay = blob_layout(table.geom)
    bits, gs, _ = table.geom
    per_expert = 0
    for role in ("gate", "up"):
        rows, cols = lay[role][2], lay[role][3]
        per_expert += rows * cols * bits // 8 + rows * (cols // gs) * table.blobs[0]["flat"]["scale"].element_size()
    return per_expert * len(set(idx.reshape(-1).tolist()))


def prefill_bench(args, device):
    """Configuration 2 through the tcgen05 grouped-GEMM path: one layer call of 2048 tokens per
    step (top-2 over 8 experts, logits skewed so expert loads differ ~4x), two layers rotated."""
    import ctypes

    import vaayu_b200 as vb
    from vaayu_b200 import packed_expert_kernels as pk
    from vaayu_b200 import synthetic
    wl = PREFILL
    T, K, H, I = wl["tokens"], wl["top_k"], wl["hidden"], wl["inter"]
    L = 2
    layers = [pk.ExpertTable(make_layer(2000 + l, wl, device)) for l in range(L)]
    batches = []
    for l in range(L):
        g = torch.Generator(device=device).manual_seed(20_000 + l)
        batches.append(tuple(v.to(device) for v in synthetic.make_tokens(T, H, wl["experts"], K, g,
                                                                         skew=wl["skew"])))
    loads = [torch.bincount(b[2].reshape(-1), minlength=wl["experts"]).tolist() for b in batches]
    out = torch.empty(T, H, dtype=torch.float32, device=device)
    ws = torch.empty(pk.moe_workspace_bytes(layers[0], T, K, path=vb.PATH_PREFILL), dtype=torch.uint8,
                     device=device)

    def step(i):
        x, w, idx = batches[i % L]
        vb.moe_forward(x, idx, w, layers[i % L], out=out, path=vb.PATH_PREFILL, workspace=ws)

    for i in range(max(3, args.warmup)):
        step(i)
    if args.profile:
        ms = time_steps(step, args.steps, device)
        print(json.dumps({"profile": "prefill", "ms_per_step": ms, "tokens": T, "layers": L}))
        return None
    steps = max(5, min(args.steps, 20))
    with ClockSampler(device.index or 0) as clocks:
        ms = time_steps(step, steps, device)
    flops = 2.0 * T * K * 3 * H * I
    # per-stage device times (serialised stages) for the per-kernel roofline
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    for e in evs:
        e.record()
    torch.cuda.synchronize(device)
    handles = (ctypes.c_void_p * 5)(*[e.cuda_event for e in evs])
    st = {"plan_gather": [], "gate_up_gemm": [], "down_gemm": [], "combine": []}
    for i in range(steps):
        x, w, idx = batches[i % L]
        tb = layers[i % L]
        c = pk._make_call(tb.geom_s, x, T, K, tb.n_experts, tb.table.data_ptr(), idx.data_ptr(), 6, w,
                          w.stride(0), w.stride(1), None, out, None, None)
        c.stage_events, c.n_stage_events = ctypes.cast(handles, ctypes.c_void_p), 5
        pk._enqueue(c, vb.PATH_PREFILL, device, ws)
        torch.cuda.synchronize(device)
        st["plan_gather"].append(evs[0].elapsed_time(evs[1]))
        st["gate_up_gemm"].append(evs[1].elapsed_time(evs[2]))
        st["down_gemm"].append(evs[2].elapsed_time(evs[4]))
        st["combine"].append(evs[4].elapsed_time(evs[3]))
    st = {k: statistics.mean(v) for k, v in st.items()}
    burst, sustained, src = bf16_peak()
    gu_tf = (2.0 * T * K * 2 * H * I) / (st["gate_up_gemm"] / 1e3) / 1e12
    dn_tf = (2.0 * T * K * H * I) / (st["down_gemm"] / 1e3) / 1e12
    traffic = None
    tfile = ROOT / "profiles" / "prefill_gemm_traffic.json"
    if tfile.exists():
        try:
            traffic = json.loads(tfile.read_text()).get("bytes_per_launch")
        except Exception:
            traffic = None
    layer_tf = flops / (ms / 1e3) / 1e12
    cpu = cpu_prefill_baseline(layers[0], batches[0]) if not args.no_cpu else None
    return {
        "workload": wl["name"], "tokens": T, "top_k": K, "experts": wl["experts"], "hidden": H,
        "expert_intermediate": I, "group_size": wl["group"], "layers_rotated": L,
        "expert_rows_per_layer": loads,
        "load_ratio_max_min": statistics.mean(max(x) / max(1, min(x)) for x in loads),
        "l2": "inputs larger than L2: each step reads ~730 MB of expert weights",
        "tokens_per_s": T / (ms / 1e3), "ms_per_step": ms, "steps": steps,
        "layer_tflops": layer_tf, "layer_frac_of_bf16_burst": layer_tf / burst,
        "algorithmic_flops_per_step": flops,
        "roofline": {"kernel": "gemm_kernel<gate/up> (tcgen05, int4 dequant in shared memory)",
                     "bound": "tensor", "achieved": gu_tf, "peak": burst, "unit": "TFLOP/s",
                     "frac": gu_tf / burst, "peak_source": src + " (burst)",
                     "frac_of_sustained": gu_tf / sustained if sustained else None,
                     "traffic": traffic, "launch_ms": st["gate_up_gemm"]},
        "down_gemm": {"achieved_tflops": dn_tf, "frac": dn_tf / burst, "launch_ms": st["down_gemm"]},
        "stage_ms": st,
        "cpu_baseline": cpu,
        "gpu_launches": 5 * steps,
        "clocks": clocks.summary(),
    }


def block_scaled_bench(args, device):
    """Configuration 4: FP8-e4m3 [4096, 14336] with an fp32 scale per 128 x 128 block and NVFP4
    (e2m1, an e4m3 scale per 16) of the same shape, each dequantised to bf16 and fused into a
    decode GEMV at batch 1 and 16.  Two weight copies rotate so every call reads from HBM."""
    from vaayu_b200 import block_scaled as bs
    N, K, g, fp8, fp4 = cfg4_weights(device)
    peak, src = hbm_peak()
    steps = max(5, min(args.steps, 20))
    res = {}

    def timed(fn, nbytes):
        for i in range(3):
            fn(i)
        ms = time_steps(fn, steps, device)
        gbs = nbytes / (ms / 1e3) / 1e9
        return {"ms": ms, "GBps": gbs, "frac": gbs / peak}

    out_bytes = N * K * 2
    res["fp8_dequant"] = timed(lambda i: bs.dequantize_block_scaled(*fp8[i % 2]),
                               N * K + fp8[0][1].numel() * 4 + out_bytes)
    res["fp4_dequant"] = timed(lambda i: bs.dequantize_fp4_block_scaled(*fp4[i % 2]),
                               N * K // 2 + N * K // 16 + out_bytes)
    for t in (1, 16):
        x = torch.randn(t, K, generator=g, device=device).to(torch.bfloat16)
        o = torch.empty(t, N, dtype=torch.bfloat16, device=device)
        res[f"fp8_gemv_T{t}"] = timed(lambda i: bs.fp8_gemv(x, *fp8[i % 2], out=o),
                                      N * K + fp8[0][1].numel() * 4 + t * (K + N) * 2)
        res[f"fp4_gemv_T{t}"] = timed(lambda i: bs.fp4_gemv(x, *fp4[i % 2], out=o),
                                      N * K // 2 + N * K // 16 + t * (K + N) * 2)
    return {"workload": "cfg4: block-scaled FP8 / NVFP4 [4096, 14336] dequant and decode GEMV",
            "bound": "hbm", "peak_GBps": peak, "peak_source": src,
            "bytes": "weights + scales read, bf16 output written (dequant) / x read, out written (GEMV)",
            "steps": steps, "results": res, "gpu_launches": 6 * steps}


def cfg4_weights(device, copies=2):
    """Configuration 4's weights: [4096, 14336] FP8-e4m3 with an fp32 scale per 128 x 128 block and
    NVFP4 (random e2m1 codes, an e4m3 scale per 16), `copies` of each, seeded."""
    N, K = 4096, 14336
    g = torch.Generator(device=device).manual_seed(4)
    fp8, fp4 = [], []
    for _ in range(copies):
        w = torch.randn(N, K, generator=g, device=device)
        amax = w.abs().reshape(N // 128, 128, K // 128, 128).amax(dim=(1, 3)).clamp_min(1e-6)
        scale = (amax / 448.0).float()
        q = (w / scale.repeat_interleave(128, 0).repeat_interleave(128, 1)).to(torch.float8_e4m3fn)
        fp8.append((q, scale))
        codes = torch.randint(0, 256, (N, K // 2), generator=g, device=device, dtype=torch.int32).to(torch.uint8)
        sc = (torch.rand(N, K // 16, generator=g, device=device) * 2 + 0.25).to(torch.float8_e4m3fn)
        fp4.append((codes, sc))
        del w, q
    return N, K, g, fp8, fp4


def gemv_profile(device):
    """Three FP8 then three FP4 configuration-4 GEMVs at batch 1, then three FP8 and three FP4
    dequantisations (the launches an ncu capture reads)."""
    from vaayu_b200 import block_scaled as bs
    N, K, g, fp8, fp4 = cfg4_weights(device, copies=1)
    x = torch.randn(1, K, generator=g, device=device).to(torch.bfloat16)
    o = torch.empty(1, N, dtype=torch.bfloat16, device=device)
    for _ in range(3):
        bs.fp8_gemv(x, *fp8[0], out=o)
    for _ in range(3):
        bs.fp4_gemv(x, *fp4[0], out=o)
    for _ in range(3):
        bs.dequantize_block_scaled(*fp8[0])
    for _ in range(3):
        bs.dequantize_fp4_block_scaled(*fp4[0])
    torch.cuda.synchronize(device)
    print(json.dumps({"profile": "gemv", "n": N, "k": K, "tokens": 1}))


def record_layout(tensors):
    """One step's input tensors packed into a single byte record (each field 16-byte aligned):
    the record size, and a function giving a uint8 record's views as those tensors."""
    fields = [(t.dtype, t.shape, t.numel() * t.element_size()) for t in tensors]
    offs, nbytes = [], 0
    for _, _, nb in fields:
        offs.append(nbytes)
        nbytes += -(-nb // 16) * 16

    def views(buf):
        return [buf[o:o + nb].view(dt).view(shp) for o, (dt, shp, nb) in zip(offs, fields)]
    return nbytes, views


def pinned_record(tensors, nbytes, views):
    rec = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    for v, src in zip(views(rec), tensors):
        v.copy_(src.cpu())
    return rec


def time_steps(fn, steps, device):
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(steps):
        fn(i)
    end.record()
    torch.cuda.synchronize(device)
    return start.elapsed_time(end) / steps


def static_config(wl, world, layers, mode):
    """The workload description shared by both arms' JSON lines (no run-time measurements)."""
    T, E = wl["tokens"], wl["experts"]
    cfg = {"workload": wl["name"], "hidden": wl["hidden"], "expert_intermediate": wl["inter"],
           "experts": E, "top_k": wl["top_k"], "group_size": wl["group"], "layers_rotated": layers,
           "zero_points": bool(wl.get("zeros")), "shared_experts": wl.get("shared", 0)}
    if mode == "decode":
        cfg["tokens_per_gpu"] = T
        cfg["l2"] = f"inputs larger than L2: steps rotate over {layers} layers, each step reads its routed experts' weights"
        cfg["parallelism"] = ("ep1" if world == 1 else
                              f"ep{world}: {E // world} experts per GPU; replicate mode (one NCCL all-gather of "
                              f"the tokens, one all-to-all of per-token partial sums, rank-ordered combine)")
    else:
        cfg["tokens_total"] = T
        cfg["tokens_per_gpu"] = T // world
        if wl.get("skew"):
            cfg["router_skew"] = f"logits + linspace(0, {wl['skew']}, {E})"
        cfg["l2"] = f"inputs larger than L2: steps rotate over {layers} layers of {E} experts"
        cfg["parallelism"] = ("ep1" if world == 1 else
                              f"ep{world}: {E // world} experts per GPU ({wl.get('placement', 'contiguous')}); "
                              f"dispatch mode (bounded-capacity all-to-alls of rows and contributions, "
                              f"ascending-global-expert combine)")
    return cfg


def staged_call(table, x, ids, w, device, path, workspace, stage_names, **kw):
    """One moe_forward-equivalent call with the library's per-stage events: {stage: ms}."""
    import ctypes

    from vaayu_b200 import packed_expert_kernels as pk
    n = 5 if path == 1 else 4
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
    for e in evs:
        e.record()                      # torch creates the CUDA event on its first record
    torch.cuda.synchronize(device)
    handles = (ctypes.c_void_p * n)(*[e.cuda_event for e in evs])
    T, K = ids.shape
    out = kw.pop("out", None)
    contrib = kw.pop("contrib", None)
    c = pk._make_call(table.geom_s, x, T, K, table.n_experts, table.table.data_ptr(), ids.data_ptr(),
                      6 if ids.dtype == torch.int64 else 5, w, w.stride(0), w.stride(1), None, out, contrib, None)
    c.ids_row_stride = ids.stride(0)
    for k, v in kw.items():
        setattr(c, k, v)
    c.stage_events, c.n_stage_events = ctypes.cast(handles, ctypes.c_void_p), n
    pk._enqueue(c, path, device, workspace)
    torch.cuda.synchronize(device)
    marks = [0, 1, 2, 4, 3] if path == 1 else [0, 1, 2, 3]
    return {name: evs[marks[i]].elapsed_time(evs[marks[i + 1]]) for i, name in enumerate(stage_names)}


# ── expert-parallel arms (N GPUs of one node; also configuration 3 on one GPU) ─────────────────

def _rank0_decode_roofline(layer, wl, world, device):
    """Rank 0's gate/up kernel over its last gathered batch, timed alone with the library's stage
    events: (achieved GB/s over the local routed experts' gate/up bytes + the gathered x, stages)."""
    b = next(v for k, v in layer._bufs.items() if not (isinstance(k, tuple) and k and k[0] == "dispatch"))
    T, K, H = wl["tokens"], wl["top_k"], wl["hidden"]
    xb = b["xb"]
    xa = b["recv"][:, :xb].view(torch.bfloat16)
    ga = b["recv"][:, xb:xb + 4 * K].view(torch.int32)
    wa = b["recv"][:, xb + 4 * K:xb + 4 * K + b["wb"]].view(torch.float32)
    part = torch.empty(world * T, H, dtype=torch.float32, device=device)
    st = staged_call(layer.table, xa, ga, wa, device, 0, b["ws"], ("plan", "gate_up", "down"), out=part,
                     expert_base=layer.lo, col_blocks=b["nb"])
    local = sorted({int(e) - layer.lo for e in ga.reshape(-1).tolist() if layer.lo <= int(e) < layer.lo + layer.per_rank})
    gu_bytes = gate_up_bytes(layer.table, torch.tensor(local, dtype=torch.int64)) + world * T * H * 2
    return gu_bytes / (st["gate_up"] / 1e3) / 1e9, st


def _capture_steps(L, layer_step, rank, device):
    """One CUDA graph per layer step (their collectives included); [] when capture fails here."""
    graphs = []
    try:
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
    return graphs


def _device_record(batches, device):
    """Each layer's inputs as views of one device record (the end-to-end step fills it with one
    copy): (record bytes, the views function, the records, each record's views)."""
    nbytes, views = record_layout(batches[0])
    drecs = [torch.empty(nbytes, dtype=torch.uint8, device=device) for _ in batches]
    dviews = []
    for rec, b in zip(drecs, batches):
        vs = views(rec)
        for v, src in zip(vs, b):
            v.copy_(src)
        dviews.append(vs)
    return nbytes, views, drecs, dviews


def run_ep_decode(args, rank, world, local, wl):
    """`wl` (configuration 1 or 3) at `wl['tokens']` tokens per rank (weak scaling), the routed
    experts sharded E/N per rank, steps rotating over `args.layers` layers, each layer step one CUDA
    graph.  A workload with `shared` experts replicates them on every rank, applies them to the
    rank's own tokens and adds their output in bf16 (the model epilogue: out.to(bf16) +
    shared.to(bf16)); on one GPU the shared expert rides in the layer call."""
    from vaayu_b200.ep import ExpertParallelLayer
    from vaayu_b200.packed_expert_kernels import (PATH_DECODE, ExpertTable, _with_shared, moe_forward_with_shared,
                                                  moe_workspace_bytes, shared_expert_forward)
    device = torch.device("cuda", local)
    E, T, K, H = wl["experts"], wl["tokens"], wl["top_k"], wl["hidden"]
    per = E // world
    L = args.layers
    layers = [ExpertParallelLayer(make_layer(1000 * l, wl, device, (rank * per, (rank + 1) * per)), E,
                                  col_blocks=getattr(args, "ep_col_blocks", None)) for l in range(L)]
    batches = [tuple(v.to(device) for v in make_tokens(l * 97 + rank, wl, T, device)) for l in range(L)]
    out = torch.empty(T, H, dtype=torch.float32, device=device)
    shared = None
    if wl.get("shared"):
        shared = [ExpertTable(make_layer(5000 + l, dict(wl, experts=1), device)) for l in range(L)]
        sh_out = torch.empty(T, H, dtype=torch.float32, device=device)
        sh_ws = torch.empty(moe_workspace_bytes(shared[0], T, 1, path=PATH_DECODE), dtype=torch.uint8, device=device)
        result = torch.empty(T, H, dtype=torch.bfloat16, device=device)
        if world == 1:
            fused_ws = torch.empty(moe_workspace_bytes(_with_shared(layers[0].table, shared[0]), T, K + 1,
                                                       path=PATH_DECODE), dtype=torch.uint8, device=device)

    def layer_step(l, x, w, idx):       # the device record's views: activations, weights, ids
        if shared is not None and world == 1:
            moe_forward_with_shared(x, idx, w, layers[l].table, shared[l], out=out, result=result,
                                    path=PATH_DECODE, workspace=fused_ws)
            return
        layers[l].forward(x, idx, w, out)
        if shared is not None:
            shared_expert_forward(x, shared[l], out=sh_out, workspace=sh_ws)
            torch.add(out.to(torch.bfloat16), sh_out.to(torch.bfloat16), out=result)

    nbytes, views, drecs, dviews = _device_record(batches, device)
    for l in range(L):
        for _ in range(2):
            layer_step(l, *dviews[l])
    torch.cuda.synchronize(device)
    barrier(world)
    graphs = _capture_steps(L, lambda l: layer_step(l, *dviews[l]), rank, device)
    barrier(world)

    def step(i):
        graphs[i % L].replay() if graphs else layer_step(i % L, *dviews[i % L])

    for i in range(args.warmup):
        step(i)
    barrier(world)
    with ClockSampler(local) as clocks:
        ms = time_steps(step, args.steps, device)
    barrier(world)
    ms = max_over_ranks(ms, world)

    pin = [pinned_record(b, nbytes, views) for b in batches]
    out_h = torch.empty(T, H, dtype=torch.float32 if shared is None else torch.bfloat16).pin_memory()

    def e2e_step(i):
        drecs[i % L].copy_(pin[i % L], non_blocking=True)
        step(i)
        out_h.copy_(out if shared is None else result, non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    barrier(world)
    e2e_ms = max_over_ranks(time_steps(e2e_step, args.steps, device), world)
    barrier(world)
    used_graphs = bool(graphs)
    del graphs               # graphs holding NCCL calls go before the process group does
    torch.cuda.synchronize(device)
    peak, peak_kind = hbm_peak()
    roof, cpu, st = None, None, None
    if rank == 0:
        if world > 1:
            achieved, st = _rank0_decode_roofline(layers[0], wl, world, device)
        else:               # the routed layer alone (the shared expert's slot left out)
            x0, w0, i0 = dviews[0]
            st = staged_call(layers[0].table, x0, i0, w0, device, 0, None, ("plan", "gate_up", "down"), out=out)
            achieved = (gate_up_bytes(layers[0].table, i0) + T * H * 2) / (st["gate_up"] / 1e3) / 1e9
        roof = {"kernel": "gate_up_kernel (rank 0, its gathered batch)", "bound": "hbm", "achieved": achieved,
                "peak": peak, "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_kind,
                "traffic": None, "launch_ms": st["gate_up"]}
        if not args.no_cpu:
            full = ExpertTable(make_layer(0, wl, device)) if world > 1 else layers[0].table
            cpu = cpu_baseline(full, make_tokens(0, wl, T, device), wl)
            del full
    uniq = statistics.mean(len(set(b[2].reshape(-1).tolist())) for b in batches)
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": T * world / (ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int4 weights, bf16 activations, fp32 accumulate",
            "data": "synthetic (seeded; int4 codes U{0..15}, fp16 scales U(0.005,0.02), x~N(0,1))",
            "config": static_config(wl, world, L, "decode"),
            "run": {"routed_experts_per_rank_batch": uniq, "cuda_graphs": used_graphs, "stage_ms": st},
            "e2e": {"value": T * world / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": out_h.numel() * out_h.element_size(),
                    "ms_per_step": e2e_ms},
            "roofline": roof,
            "cpu_baseline": cpu,
            # plan, gate/up, down and the rank-ordered sum (one GPU: the layer's combine), plus the
            # separate shared-expert call's four on several GPUs
            "gpu_launches": (4 + (4 if shared is not None and world > 1 else 0)) * args.steps,
            "clocks": clocks.summary(),
        }))


def run_ep_prefill(args, rank, world, local, wl):
    """A prefill workload at any N (strong scaling): `wl['tokens']` tokens in total, rank r holding
    tokens [r T/N, (r + 1) T/N) and its share of the experts (`wl['placement']`); dispatch mode --
    the rows to their experts' ranks by bounded-capacity all-to-alls (no host round trip after the
    first call), the local tcgen05 prefill GEMMs, contributions back by the reverse all-to-all, the
    ascending-global-expert combine on each token's home rank.  A `shared` expert runs on each rank's
    own tokens (prefill kernels) and joins in bf16.  Each layer step is one CUDA graph."""
    from vaayu_b200 import synthetic
    from vaayu_b200.ep import ExpertParallelLayer
    from vaayu_b200.packed_expert_kernels import PATH_PREFILL, ExpertTable, moe_forward, moe_workspace_bytes
    device = torch.device("cuda", local)
    E, T, K, H, I = wl["experts"], wl["tokens"], wl["top_k"], wl["hidden"], wl["inter"]
    if E % world or T % world:
        raise ValueError(f"{wl['name']} splits {E} experts and {T} tokens evenly: not over {world} GPUs")
    per, tl = E // world, T // world
    L = 2
    placement = wl.get("placement", "contiguous")
    keep = range(rank, E, world) if placement == "interleaved" else range(rank * per, (rank + 1) * per)
    layers = [ExpertParallelLayer(make_layer(2000 + l, wl, device, keep=keep), E, mode="dispatch",
                                  placement=placement, path=PATH_PREFILL) for l in range(L)]
    batches = []
    for l in range(L):
        g = torch.Generator(device=device).manual_seed(20_000 + l)
        x, w, idx = synthetic.make_tokens(T, H, E, K, g, skew=wl.get("skew", 0.0))
        sl = slice(rank * tl, (rank + 1) * tl)
        batches.append((x[sl].contiguous(), w[sl].contiguous(), idx[sl].contiguous()))
    out = torch.empty(tl, H, dtype=torch.float32, device=device)
    shared = None
    if wl.get("shared"):
        shared = [ExpertTable(make_layer(5000 + l, dict(wl, experts=1), device)) for l in range(L)]
        sh_ids = torch.zeros(tl, 1, dtype=torch.int32, device=device)
        sh_w = torch.ones(tl, 1, dtype=torch.float32, device=device)
        sh_out = torch.empty(tl, H, dtype=torch.float32, device=device)
        sh_ws = torch.empty(moe_workspace_bytes(shared[0], tl, 1, path=PATH_PREFILL), dtype=torch.uint8, device=device)
        result = torch.empty(tl, H, dtype=torch.bfloat16, device=device)
    nbytes, views, drecs, dviews = _device_record(batches, device)

    def layer_step(l):
        xv, wv, iv = dviews[l]
        layers[l].forward(xv, iv, wv, out)
        if shared is not None:
            moe_forward(xv, sh_ids, sh_w, shared[l], out=sh_out, path=PATH_PREFILL, workspace=sh_ws)
            torch.add(out.to(torch.bfloat16), sh_out.to(torch.bfloat16), out=result)

    for l in range(L):
        for _ in range(2):
            layer_step(l)
    torch.cuda.synchronize(device)
    barrier(world)
    graphs = _capture_steps(L, layer_step, rank, device)
    barrier(world)

    def step(i):
        graphs[i % L].replay() if graphs else layer_step(i % L)

    for i in range(max(3, args.warmup)):
        step(i)
    steps = max(5, min(args.steps, 20))
    barrier(world)
    with ClockSampler(local) as clocks:
        ms = time_steps(step, steps, device)
    barrier(world)
    ms = max_over_ranks(ms, world)

    pin = [pinned_record(b, nbytes, views) for b in batches]
    out_h = torch.empty(tl, H, dtype=torch.float32 if shared is None else torch.bfloat16).pin_memory()

    def e2e_step(i):
        drecs[i % L].copy_(pin[i % L], non_blocking=True)
        step(i)
        out_h.copy_(out if shared is None else result, non_blocking=True)

    for i in range(3):
        e2e_step(i)
    barrier(world)
    e2e_ms = max_over_ranks(time_steps(e2e_step, steps, device), world)
    barrier(world)
    used_graphs = bool(graphs)
    del graphs               # graphs holding NCCL calls go before the process group does
    torch.cuda.synchronize(device)
    overflow = any(ly.overflowed() for ly in layers)
    flops = 2.0 * T * (K + wl.get("shared", 0)) * 3 * H * I
    burst, sustained, src = bf16_peak()
    roof, cpu, st = None, None, None
    if rank == 0:
        # rank 0's own gate/up GEMM over the rows it received in the last step, timed alone
        ly = layers[(steps - 1) % L]
        cap = ly._caps.get((tl, K), tl * K)
        b = next(v for k, v in ly._bufs.items() if isinstance(k, tuple) and k and k[0] == "dispatch" and v["cap"] == cap)
        rx, rid, rw = b["recv_x"], b["recv_id"].view(-1, 1), b["recv_w"].view(-1, 1)
        st = staged_call(ly.table, rx, rid, rw, device, PATH_PREFILL, None,
                         ("plan_gather", "gate_up_gemm", "down_gemm", "combine"), contrib=b["contrib"])
        rows = int((rid >= 0).sum().item())
        gu_tf = 2.0 * rows * 2 * H * I / (st["gate_up_gemm"] / 1e3) / 1e12
        roof = {"kernel": "gemm_kernel<gate/up> (rank 0, the rows it received)", "bound": "tensor",
                "achieved": gu_tf, "peak": burst, "unit": "TFLOP/s", "frac": gu_tf / burst,
                "peak_source": f"{src} (burst)", "frac_of_sustained": gu_tf / sustained if sustained else None,
                "traffic": None, "launch_ms": st["gate_up_gemm"], "rows": rows}
        if not args.no_cpu:
            full = ExpertTable(make_layer(2000, wl, device))
            cpu = cpu_prefill_baseline(full, batches[0], tokens=16)
            del full
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": T / (ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": steps, "warmup": max(3, args.warmup), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int4 weights, bf16 activations, fp32 accumulate",
            "data": "synthetic (seeded; int4 codes U{0..15}, fp16 scales U(0.005,0.02), x~N(0,1))",
            "config": static_config(wl, world, L, "prefill"),
            "run": {"cuda_graphs": used_graphs, "dispatch_capacity_per_destination": layers[0]._caps.get((tl, K)),
                    "dispatch_overflowed": overflow, "layer_tflops_per_gpu": flops / (ms / 1e3) / 1e12 / world,
                    "stage_ms_rank0": st},
            "e2e": {"value": T / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": nbytes,
                    "d2h_bytes_per_step": out_h.numel() * out_h.element_size(), "ms_per_step": e2e_ms},
            "roofline": roof,
            "cpu_baseline": cpu,
            # plan, gather, gate/up GEMM, down GEMM (contributions), the dispatch plan and pack, the
            # home-rank combine (+ the shared expert's five)
            "gpu_launches": (7 + (5 if shared is not None else 0)) * steps,
            "clocks": clocks.summary(),
        }))


def run_ours(args, rank, world, local):
    import vaayu_b200 as vb
    from vaayu_b200 import packed_expert_kernels as pk
    device = torch.device("cuda", local)
    wl = dict(WORKLOAD)
    T, K = wl["tokens"], wl["top_k"]
    if args.workload == "cfg2":
        return run_ep_prefill(args, rank, world, local, dict(PREFILL, placement="interleaved"))
    if args.workload == "cfg3-prefill":
        return run_ep_prefill(args, rank, world, local, CFG3_PREFILL)
    if world > 1 or args.workload == "cfg3":
        return run_ep_decode(args, rank, world, local, CFG3 if args.workload == "cfg3" else wl)
    if args.profile == "prefill":
        return prefill_bench(args, device)
    if args.profile == "gemv":
        return gemv_profile(device)

    if args.profile and args.tokens:
        T = wl["tokens"] = args.tokens        # profiling only: the headline batch is the workload's
    layers = [pk.ExpertTable(make_layer(1000 * l, wl, device)) for l in range(args.layers)]
    batches = {}
    for t in sorted({T, 1, 8}):
        batches[t] = [tuple(v.to(device) for v in make_tokens(l, wl, t, device)) for l in range(args.layers)]
    out = torch.empty(T, wl["hidden"], dtype=torch.float32, device=device)
    # one workspace for every batch size run below (a few-token call may take split-K partials)
    ws = torch.empty(max(pk.moe_workspace_bytes(layers[0], t, K) for t in (T, 1, 8)), dtype=torch.uint8,
                     device=device)
    L = args.layers

    def step_for(t):
        bt = batches[t]
        o = out[:t]

        def step(i):
            x, w, idx = bt[i % L]
            vb.moe_forward(x, idx, w, layers[i % L], out=o, path=vb.PATH_DECODE, workspace=ws)
        return step

    def replayed(t):
        """The step at batch t replayed from one CUDA graph per layer (the way a serving loop runs
        decode: no host submission cost in the device-timed loop); eager when capture fails."""
        st = step_for(t)
        for i in range(3):
            st(i)
        graphs = _capture_steps(L, st, 0, device)
        return (lambda i: graphs[i % L].replay()) if graphs else st, bool(graphs)

    def timed_run(t, steps):
        """ms per step of `steps` consecutive layer steps at batch t, captured as ONE CUDA graph
        and replayed once (a decode step of a many-layer model replays one graph: no host
        submission and no per-layer graph launch in the timed region); per-layer replay when
        that capture fails.  Exactly `steps` layer steps are timed."""
        st = step_for(t)
        for i in range(3):
            st(i)
        run = _capture_steps(1, lambda _l: [st(i) for i in range(steps)], 0, device)
        if not run:
            rep, _ = replayed(t)
            return time_steps(rep, steps, device)
        run[0].replay()                      # warm
        ms = time_steps(lambda _i: run[0].replay(), 1, device) / steps
        del run
        return ms

    main_step, used_graphs = replayed(T)
    for i in range(args.warmup):
        main_step(i)
    if args.profile:
        # a short fixed loop of the main step for profilers: no sweep, e2e or CPU baseline
        ms = time_steps(main_step, args.steps, device)
        print(json.dumps({"profile": True, "ms_per_step": ms, "tokens": T, "layers": L}))
        return
    barrier(world)
    with ClockSampler(local) as clocks:
        ms = timed_run(T, args.steps)
    barrier(world)
    ms = max_over_ranks(ms, world)
    value = T * world / (ms / 1e3)

    # per-stage timing (serialised stages): the gate/up kernel's own duration for the roofline
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    for e in evs:
        e.record()                      # torch creates the CUDA event on its first record
    torch.cuda.synchronize(device)
    import ctypes
    handles = (ctypes.c_void_p * 4)(*[e.cuda_event for e in evs])
    stage = {"plan": [], "gate_up": [], "down": []}
    for i in range(max(3, min(args.steps, 20))):
        x, w, idx = batches[T][i % L]
        c = pk._make_call(layers[i % L].geom_s, x, T, K, layers[i % L].n_experts,
                          layers[i % L].table.data_ptr(), idx.data_ptr(), 6, w, w.stride(0),
                          w.stride(1), None, out, None, None)
        c.stage_events, c.n_stage_events = ctypes.cast(handles, ctypes.c_void_p), 4
        pk._enqueue(c, vb.PATH_DECODE, device, ws)
        torch.cuda.synchronize(device)
        stage["plan"].append(evs[0].elapsed_time(evs[1]))
        stage["gate_up"].append(evs[1].elapsed_time(evs[2]))
        stage["down"].append(evs[2].elapsed_time(evs[3]))
    gu_ms = statistics.mean(stage["gate_up"])
    gu_bytes = statistics.mean(gate_up_bytes(layers[l], batches[T][l][2]) + T * wl["hidden"] * 2
                               for l in range(L))
    peak, peak_kind = hbm_peak()
    achieved = gu_bytes / (gu_ms / 1e3) / 1e9
    layer_bytes = statistics.mean(unique_bytes(layers[l], batches[T][l][2])[0] + T * wl["hidden"] * 6
                                  for l in range(L))
    uniq = statistics.mean(unique_bytes(layers[l], batches[T][l][2])[1] for l in range(L))
    traffic = None
    tfile = ROOT / "profiles" / "gate_up_traffic.json"
    if tfile.exists():
        try:
            traffic = json.loads(tfile.read_text()).get("bytes_per_launch")
        except Exception:
            traffic = None

    # sweep: batch 1 and 8 (device-timed the same way)
    sweep = {}
    for t in (1, 8):
        m = timed_run(t, args.steps)
        b = statistics.mean(unique_bytes(layers[l], batches[t][l][2])[0] for l in range(L))
        sweep[f"T={t}"] = {"tokens_per_s": t / (m / 1e3), "ms_per_step": m,
                           "layer_GBps": b / (m / 1e3) / 1e9}

    # end to end through the public API with host buffers: each step's activations, routing
    # weights and expert ids sit in one pinned host record (16-byte aligned fields) that is copied
    # to the device in one transfer; the fp32 result is read back in full
    nbytes, views = record_layout(batches[T][0])
    pin = [pinned_record(b, nbytes, views) for b in batches[T]]
    drec = torch.empty(nbytes, dtype=torch.uint8, device=device)
    dx, dw, di = views(drec)
    out_h = torch.empty(T, wl["hidden"], dtype=torch.float32).pin_memory()

    def e2e_step(i):
        drec.copy_(pin[i % L], non_blocking=True)
        vb.moe_forward(dx, di, dw, layers[i % L], out=out, path=vb.PATH_DECODE, workspace=ws)
        out_h.copy_(out, non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    e2e_ms = max_over_ranks(time_steps(e2e_step, args.steps, device), world)
    h2d = nbytes                      # the record copied each step (its fields padded to 16 bytes)
    d2h = out_h.numel() * out_h.element_size()

    # the same step with explicit zero points (asymmetric int4, z ~ U{0..15} per row and group; the
    # headline keeps the reference's symmetric format)
    zl = [pk.ExpertTable(make_layer(1000 * l, dict(wl, zeros=True), device)) for l in range(L)]
    zstep = lambda i: vb.moe_forward(batches[T][i % L][0], batches[T][i % L][2], batches[T][i % L][1], zl[i % L],
                                     out=out, path=vb.PATH_DECODE, workspace=ws)
    for i in range(3):
        zstep(i)
    zms = time_steps(zstep, args.steps, device)
    zb = statistics.mean(unique_bytes(zl[l], batches[T][l][2])[0] for l in range(L))
    sweep[f"T={T}, zero points"] = {"tokens_per_s": T / (zms / 1e3), "ms_per_step": zms,
                                    "layer_GBps": zb / (zms / 1e3) / 1e9}
    del zl

    cpu = cpu_baseline(layers[0], batches[T][0], wl) if rank == 0 and not args.no_cpu else None
    del layers, batches
    torch.cuda.empty_cache()
    prefill = prefill_bench(args, device) if not args.no_prefill else None
    blocks = block_scaled_bench(args, device) if not args.no_prefill else None
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int4 weights, bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded; int4 codes U{0..15}, fp16 scales U(0.005,0.02), x~N(0,1))",
        "config": static_config(wl, world, L, "decode"),
        "run": {"unique_experts_per_step": uniq, "expert_weight_MB_per_step": layer_bytes / 1e6,
                "cuda_graphs": used_graphs,
                "timing": "value and sweep: K consecutive layer steps captured as one CUDA graph, replayed once"},
        "e2e": {"value": T * world / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "roofline": {"kernel": "gate_up_kernel", "bound": "hbm", "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_kind,
                     "traffic": traffic, "algorithmic_bytes_per_launch": gu_bytes,
                     "launch_ms": gu_ms},
        "layer": {"GBps": layer_bytes / (ms / 1e3) / 1e9, "frac_of_hbm": layer_bytes / (ms / 1e3) / 1e9 / peak,
                  "stage_ms": {k: statistics.mean(v) for k, v in stage.items()}},
        "sweep": sweep,
        "cpu_baseline": cpu,
        "gpu_launches": 4 * args.steps,   # plan, gate/up, down, ordered combine per step
        "clocks": clocks.summary(),
        "prefill": prefill,
        "block_scaled": blocks,
    }
    if rank == 0:
        print(json.dumps(line))


# ── the CPU side: oracle port of the reference's path ───────────────────────────────────────

def _oracle_inputs(table, batch):
    from tests import helpers as H
    experts = [H.oracle_expert(b) for b in table.blobs]
    x, w, idx = batch
    return experts, H.to_np(x), H.to_np(idx), w.cpu().numpy()


def cpu_baseline(table, batch, wl, budget_s=10.0):
    from oracle import oracle as O
    experts, x, idx, w = _oracle_inputs(table, batch)
    threads = os.cpu_count() or 1
    O.moe_layer(table.geom, experts, x, O.BF16, idx, w, O.F32, O.F16, threads=threads)
    reps, t0 = 0, time.perf_counter()
    while True:
        O.moe_layer(table.geom, experts, x, O.BF16, idx, w, O.F32, O.F16, threads=threads)
        reps += 1
        if time.perf_counter() - t0 >= budget_s or reps >= 200:
            break
    el = time.perf_counter() - t0
    return {"value": reps * x.shape[0] / el, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{reps} full layer calls of the benchmark workload ({x.shape[0]} tokens each, "
                      f"{el:.1f} s), C oracle restating stock_experts_prefill(linear=_linear_fp32)"}


def cpu_prefill_baseline(table, batch, tokens=48):
    """The oracle port on a bounded sample of configuration 2: the first `tokens` tokens."""
    from oracle import oracle as O
    x, w, idx = batch
    experts, xs, ids, ws = _oracle_inputs(table, (x[:tokens], w[:tokens], idx[:tokens]))
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    O.moe_layer(table.geom, experts, xs, O.BF16, ids, ws, O.F32, O.F16, threads=threads)
    el = time.perf_counter() - t0
    return {"value": tokens / el, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"one layer call of the first {tokens} of the {x.shape[0]} tokens ({el:.1f} s), "
                      f"C oracle restating stock_experts_prefill(linear=_linear_fp32)"}


def run_reference(args, rank, world, local):
    """The reference's CPU implementation of the path (the C oracle port of
    `stock_experts_prefill(linear=_linear_fp32)`) on this host's cores, over the same layers and
    batches the default arm rotates through (rank 0's batches), with the same `config`."""
    if rank != 0:
        return
    from oracle import oracle as O
    wl = dict(WORKLOAD)
    T, L = wl["tokens"], args.layers
    device = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    calls = []
    if device.type == "cuda":
        from vaayu_b200 import packed_expert_kernels as pk
        for l in range(L):
            table = pk.ExpertTable(make_layer(1000 * l, wl, device))
            batch = make_tokens(l * 97 if world > 1 else l, wl, T, device)
            calls.append((table.geom, *_oracle_inputs(table, batch)))
            del table
        torch.cuda.empty_cache()
    else:
        import vaayu_b200 as vb
        from vaayu_b200 import synthetic

        class _Table:
            pass
        for l in range(L):
            g = torch.Generator().manual_seed(l)
            table = _Table()
            table.blobs = [vb.build_expert_blob(synthetic.make_expert(wl["hidden"], wl["inter"], g))
                           for _ in range(wl["experts"])]
            table.geom = table.blobs[0]["geom"]
            batch = synthetic.make_tokens(T, wl["hidden"], wl["experts"], wl["top_k"], g)
            calls.append((table.geom, *_oracle_inputs(table, batch)))
    threads = os.cpu_count() or 1

    def run(i):
        geom, experts, x, idx, w = calls[i % L]
        O.moe_layer(geom, experts, x, O.BF16, idx, w, O.F32, O.F16, threads=threads)

    for i in range(args.warmup):
        run(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        run(i)
    el = time.perf_counter() - t0
    ms = el * 1e3 / args.steps
    v = T / (ms / 1e3)
    sample = (f"{args.steps} layer calls of {T} tokens rotating over the {L} layers the default arm times "
              f"(rank 0's batches), all {threads} host threads")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int4 weights, bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded; int4 codes U{0..15}, fp16 scales U(0.005,0.02), x~N(0,1))",
        "config": static_config(wl, world, L, "decode"),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--profile", nargs="?", const="decode", choices=("decode", "prefill", "gemv"), default=None,
                    help="only the timed loop of the decode (default) or prefill step, or three FP8 then "
                         "three FP4 configuration-4 GEMVs at batch 1, for ncu")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the configuration-2 prefill measurement")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baselines")
    ap.add_argument("--tokens", type=int, default=None,
                    help="with --profile decode: the decode batch (default: the workload's)")
    ap.add_argument("--workload", default="cfg1", choices=("cfg1", "cfg2", "cfg3", "cfg3-prefill"),
                    help="cfg1 (default): the headline decode workload (expert-parallel for N > 1); "
                         "cfg2: the Mixtral-shaped 2048-token prefill, experts and tokens split over N "
                         "GPUs (strong scaling, dispatch mode); cfg3: DeepSeek-V3 shape, "
                         "expert-parallel decode at any N; cfg3-prefill: the same layer, 4096 tokens "
                         "split over N GPUs (dispatch mode)")
    ap.add_argument("--ep-col-blocks", type=int, default=None, choices=(1, 2, 4),
                    help="tokens per expert pass (x8) in the expert-parallel step; default by load")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank, world, local = dist_setup()
    try:
        if args.impl == "reference":
            run_reference(args, rank, world, local)
        else:
            run_ours(args, rank, world, local)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
