"""Fused packed-int4 MoE expert layer on B200: the operator surface of archish9/Vaayu's
vaayu/packed_expert_kernels.py, behind libvaayu_b200's sm_100a kernels.

Entry points (same names, arguments and results as the reference's):

    packed_experts_decode(x, pairs, routing_weights, out, act_fn)                  :459-480
    packed_experts_decode_graphed(layer, x, pairs, routing_weights, shared,
                                  act_fn, tail)                                    :531-654
    packed_experts_prefill(x, eidx_cpu, routing_weights, blobs, out, act_fn)       :838-861
    install_packed_expert_kernels(vaayu_ref)                                       :902-1012

plus the device-resident form the reference does not have: `ExpertTable` (a layer's resident
expert blobs as one device pointer table) and `moe_forward` (expert ids and routing weights
already on the device -- no host sync, graph-capturable).

What differs from the reference, on purpose:
  * No fallback.  A call the kernels cannot take (mixed geometries, a dense entry, unsupported
    geometry or dtype) raises NotImplementedError instead of running the stock per-expert loop:
    this build has no CPU / torch / Triton path.  `install_packed_expert_kernels` still answers
    False (and logs why) for a model it cannot serve, leaving the engine's own path in place.
  * The verdict is a geometry gate only (`_unsupported`); the first-call comparison against the
    stock arithmetic lives in the test suite, not in the product.
  * Zero-point blobs are served (see vaayu_b200.moe_patch).
  * A call's host-built table reaches the device through torch's pinned caching allocator with a
    stream-ordered copy (`_stage`); the layer graph records device work only and is fed the same
    way.  Reports go to the "vaayu_b200" logger.
Arithmetic: every weight is act(act(u - z) * act(scale)); g, u, SiLU(g), h, y are rounded to
the activation dtype where the stock loop rounds; y * w is one fp32 product (rounded to the
activation dtype when the weight is in that dtype); each token's contributions are summed in
fp32 in ascending expert id, then slot -- `accumulate_expert_outputs`' order.
"""
from __future__ import annotations

import collections
import ctypes
import functools
import gc
import logging
import os
import threading

import torch

from . import _lib
from .moe_patch import blob_layout, zero_layout

_ROLES = ("gate", "down", "up")
_DTYPE_CODE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}
PATH_DECODE, PATH_PREFILL = 0, 1
# average routed rows per expert above which moe_forward's default path is the tcgen05 prefill
PREFILL_ROWS_PER_EXPERT = 12


def _layout(geom) -> dict:
    """{role: (word offset, scale offset, rows, cols)} inside a blob's flat streams."""
    return blob_layout(geom)


def _unsupported(geom, act_dtype, scale_dtype, w_dtype):
    """The first reason the layer kernels cannot serve this (geometry, dtypes), or None."""
    bits, gs, roles = geom
    dims = {role: (rows, cols) for role, rows, cols in roles}
    if sorted(dims) != sorted(_ROLES):
        return f"the blob holds roles {sorted(dims)}; the layer kernels need exactly gate, up and down"
    inter, hid = dims["gate"]
    if dims["up"] != (inter, hid) or dims["down"] != (hid, inter):
        return f"role shapes {dims} do not form a gated MLP (gate / up [I, H], down [H, I])"
    checks = (
        (bits == 4, f"{bits}-bit codes: the layer kernels read int4"),
        (gs >= 32 and gs & (gs - 1) == 0, f"group size {gs}: a power of two of at least 32 is needed"),
        (hid % 128 == 0 and inter % 128 == 0 and hid % gs == 0 and inter % gs == 0,
         f"hidden {hid} / intermediate {inter} must be multiples of 128 and of the group size {gs}"),
        (act_dtype in (torch.bfloat16, torch.float16), f"activation dtype {act_dtype}: bf16 or fp16"),
        (scale_dtype in _DTYPE_CODE, f"scale dtype {scale_dtype}"),
        (w_dtype in _DTYPE_CODE, f"routing-weight dtype {w_dtype}"),
    )
    return next((why for ok, why in checks if not ok), None)


@functools.lru_cache(maxsize=None)
def _geom_struct(geom, scale_dtype, has_zero) -> _lib.ExpertGeom:
    bits, gs, roles = geom
    lay, zl = blob_layout(geom), zero_layout(geom)
    g = _lib.ExpertGeom()
    g.hidden, g.inter = lay["gate"][3], lay["gate"][2]
    g.bits, g.group_size = bits, gs
    g.scale_dtype = _DTYPE_CODE[scale_dtype]
    g.has_zero = int(has_zero)
    for i, role in enumerate(("gate", "up", "down")):
        g.word_off[i], g.scale_off[i] = lay[role][0], lay[role][1]
        g.zero_off[i] = zl[role] if has_zero else 0
    return g


def _blob_ptrs(blob) -> tuple:
    flat = blob["flat"]
    for name, t in flat.items():
        if t.data_ptr() % 16:
            raise RuntimeError(f"blob stream '{name}' is not 16-byte aligned")
    zero = flat.get("zero")
    return (flat["packed"].data_ptr(), flat["scale"].data_ptr(), 0 if zero is None else zero.data_ptr())


def _blob_key(blob):
    flat = blob["flat"]
    return blob["geom"], flat["scale"].dtype, "zero" in flat


# ── per-stream scratch and host-built tables ─────────────────────────────────────────────

class _Workspace:
    """Scratch for the kernels, one buffer per (device, stream), grown on demand (torch's
    caching allocator hands it out; the C ABI itself never allocates)."""

    def __init__(self):
        self._bufs: dict = {}
        self._lock = threading.Lock()

    def get(self, device, nbytes: int) -> torch.Tensor:
        key = (device, torch.cuda.current_stream(device).cuda_stream)
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
                self._bufs[key] = buf
            return buf


_WORKSPACE = _Workspace()
_VERDICTS: dict = {}
_PF_VERDICTS: dict = {}
_LAYER_VERDICTS: dict = {}     # moe_forward's (geometry, act, scale, weight dtypes) -> refusal or None


def _stage(values: torch.Tensor, device, into: "torch.Tensor | None" = None) -> torch.Tensor:
    """A host-built table on `device`: copied on the current stream from a pinned block of torch's
    caching host allocator, which keeps the block from reuse until the copy has read it.  The
    device side is a fresh caching-allocator tensor (reusable only by later work on this stream),
    or `into` when given (a graph's static table)."""
    pinned = values.pin_memory()
    if into is None:
        return pinned.to(device, non_blocking=True)
    into[:values.numel()].copy_(pinned, non_blocking=True)
    return into


# ── the call itself ──────────────────────────────────────────────────────────────────────

def _make_call(geom_s, x, n_tokens, top_k, n_experts, table_ptr, ids_ptr, ids_code, rw,
               w_tok_stride, w_slot_stride, w_index_ptr, out, contrib, h_out) -> _lib.MoeCall:
    c = _lib.MoeCall()
    gp = geom_s.__dict__.get("_pointer")            # built once per geometry struct
    if gp is None:
        gp = geom_s.__dict__["_pointer"] = ctypes.pointer(geom_s)
    c.geom = gp
    c.act_dtype = _DTYPE_CODE[x.dtype]
    c.n_experts, c.top_k, c.ids_dtype, c.n_tokens = n_experts, top_k, ids_code, n_tokens
    c.x, c.x_row_stride = x.data_ptr(), (x.stride(0) if x.dim() == 2 else x.shape[-1])
    c.expert_table, c.expert_ids = table_ptr, ids_ptr
    c.weights, c.w_dtype = rw.data_ptr(), _DTYPE_CODE[rw.dtype]
    c.w_tok_stride, c.w_slot_stride = w_tok_stride, w_slot_stride
    c.w_index = w_index_ptr
    if out is not None:
        c.out, c.out_row_stride = out.data_ptr(), (out.stride(0) if out.dim() == 2 else out.shape[-1])
    c.contrib = _lib.ptr(contrib)
    c.h_out = _lib.ptr(h_out)
    return c


def _enqueue(c: _lib.MoeCall, path: int, device, workspace: "torch.Tensor | None" = None) -> None:
    need = _lib.lib().vy_moe_workspace_size(ctypes.byref(c), path)
    if workspace is not None and workspace.numel() < need and path == PATH_DECODE and c.k_splits == 0:
        # a workspace sized for a larger batch: a few-token call then runs without split K
        c.k_splits = 1
        need = _lib.lib().vy_moe_workspace_size(ctypes.byref(c), path)
        c.k_splits = 0     # the library makes the same choice from the workspace it is given
    ws = workspace if workspace is not None else _WORKSPACE.get(device, need)
    if ws.numel() < need:
        raise RuntimeError(f"workspace of {ws.numel()} bytes, {need} needed")
    c.workspace, c.workspace_bytes = ws.data_ptr(), ws.numel()
    fn = _lib.lib().vy_moe_prefill if path == PATH_PREFILL else _lib.lib().vy_moe_decode
    _lib.check(fn(ctypes.byref(c), _lib.stream_of(device)),
               "vy_moe_prefill" if path == PATH_PREFILL else "vy_moe_decode")


def _check_x(x, what):
    if x.dim() not in (1, 2) or x.stride(-1) != 1:
        raise RuntimeError(f"{what}: activations must be [tokens, hidden] with a unit last stride")


def _pairs_table(pairs) -> torch.Tensor:
    """A one-token decode call's table payload: int64 [4n] = n x (packed, scale, zero) stream
    addresses in the pairs' order, then n int32 table indices (0..n-1: the pairs' order is the
    order the fp32 sum runs in) and n int32 routing slots."""
    n = len(pairs)
    vals = torch.empty(4 * n, dtype=torch.int64)
    vals[:3 * n] = torch.tensor([p for blob, _s in pairs for p in _blob_ptrs(blob)], dtype=torch.int64)
    tail = vals[3 * n:].view(torch.int32)
    tail[:n] = torch.arange(n, dtype=torch.int32)
    tail[n:] = torch.tensor([s for _b, s in pairs], dtype=torch.int32)
    return vals


def _decode_from_table(x, n, geom_s, dev_tbl, rw, out, h_out=None, workspace=None):
    """Launch the decode kernels over a device table laid out as `_pairs_table`."""
    tail = dev_tbl[3 * n:4 * n].view(torch.int32)
    rw_flat = rw.reshape(-1)
    c = _make_call(geom_s, x, 1, n, n, dev_tbl.data_ptr(), tail.data_ptr(), _lib.I32, rw_flat,
                   0, rw_flat.stride(0), tail[n:].data_ptr(), out, None, h_out)
    _enqueue(c, PATH_DECODE, x.device, workspace)


def _launch(x, pairs, routing_weights, out, h_out=None) -> None:
    """The decode kernels over `pairs`, into `out`.  No checks: `_checked` gates this."""
    geom_s = _geom_struct(*_blob_key(pairs[0][0]))
    tbl = _stage(_pairs_table(pairs), x.device)
    _decode_from_table(x, len(pairs), geom_s, tbl, routing_weights, out, h_out)


def _checked(x, pairs, routing_weights, act_fn=None) -> None:
    """Raises NotImplementedError when the kernels cannot take this call's (geometry, dtypes);
    the answer is cached per key."""
    blob = pairs[0][0]
    key = (blob["geom"], x.dtype, routing_weights.dtype, blob["flat"]["scale"].dtype)
    why = _VERDICTS.get(key, False)
    if why is False:
        why = _VERDICTS[key] = _unsupported(blob["geom"], x.dtype, blob["flat"]["scale"].dtype,
                                            routing_weights.dtype)
    if why is not None:
        raise NotImplementedError(f"fused packed-expert decode kernel: {why}")


def _one_geometry(entries, what):
    geoms = {(e.get("geom"), "flat" in e) for e in entries}
    if len(geoms) != 1 or any(g is None or not f for g, f in geoms):
        raise NotImplementedError(
            f"{what}: the entries are not all pack-quantized blobs of one geometry (a dense "
            "entry, a packed expert with no fused pass, or mixed formats); vaayu_b200 has no "
            "per-expert fallback for such a call")
    zs = {"zero" in e["flat"] for e in entries}
    ss = {e["flat"]["scale"].dtype for e in entries}
    if len(zs) != 1 or len(ss) != 1:
        raise NotImplementedError(f"{what}: entries mix zero-point / scale formats")


def packed_experts_decode(x, pairs, routing_weights, out, act_fn=None) -> None:
    """One token's routed-expert sum for one MoE layer, written into `out`.

    x               [1, hidden], activation dtype (bf16 / fp16), on a CUDA device
    pairs           [(blob, slot), ...] sorted by (expert id, slot): the order the fp32 sum runs
                    in; `blob` is a `build_expert_blob` entry
    routing_weights this token's [1, top_k] (or [top_k]) weights; `slot` indexes them
    out             [1, hidden] float32, overwritten
    act_fn          the experts' activation; the kernels compute SiLU (checked at install)
    """
    dev = _lib.require_cuda(x, routing_weights, out, what="packed_experts_decode")
    if not pairs:
        raise ValueError("packed_experts_decode: no routed pairs")
    _one_geometry([b for b, _s in pairs], "packed_experts_decode")
    _check_x(x, "packed_experts_decode")
    if out.dtype != torch.float32 or out.stride(-1) != 1:
        raise RuntimeError("packed_experts_decode: out must be float32 with a unit last stride")
    _checked(x, pairs, routing_weights, act_fn)
    with torch.cuda.device(dev):
        _launch(x, pairs, routing_weights, out)


# ── one CUDA graph per MoE layer for one-token decode ────────────────────────────────────
#
# A layer's graph records only device work -- the routing plan, the gate/up and down kernels, the
# combine and, on request, the forward's epilogue -- over static device buffers.  A call copies its
# pair table into the graph's static table with an ordinary stream-ordered copy (`_stage`) and
# replays.  The graph is recorded again when an input address, the pair count, the format or the
# epilogue changes.  The first graph recorded for a layer is held bitwise to an eager launch of the
# same call; a mismatch, or a recording that raises, switches the graph path off for that layer
# (its calls then return None: the caller launches eagerly).  Reasons are logged once each.

log = logging.getLogger("vaayu_b200")
GRAPH_STATS: collections.Counter = collections.Counter()   # recorded, replays, recorded_unused, off
_GRAPHS: dict = {}              # layer -> _DecodeGraph
_GRAPH_OFF: dict = {}           # layer -> why the graph path is off for it
_GRAPH_VERIFIED: set = set()    # layers whose first recording matched the eager launch bitwise
_GRAPH_NOTES: set = set()       # reasons already logged
_CAPTURE_STREAMS: dict = {}     # device -> side stream the recordings run on
_KERNELS_READY: set = set()     # devices where an eager call has set the kernels' attributes up


def _tail(out, dtype, shared):
    """The forward's epilogue: the fp32 sum cast back, plus the shared expert's output."""
    result = out.to(dtype)
    if shared is not None:
        result = result + shared.to(result.dtype)
    return result


def _graph_note(why: str) -> None:
    if why not in _GRAPH_NOTES:
        _GRAPH_NOTES.add(why)
        log.warning("vaayu_b200 decode graph: %s", why)


def _graph_off(layer, why: str) -> None:
    _GRAPH_OFF[layer] = why
    _GRAPHS.pop(layer, None)
    GRAPH_STATS["off"] += 1
    _graph_note(f"layer {layer} stays eager: {why}")


class _DecodeGraph:
    """One layer's recorded decode step and the static buffers it reads and writes."""

    def __init__(self, key, x, n_pairs, shared, tail):
        dev = x.device
        self.key, self.n, self.tail, self.replays = key, n_pairs, tail, 0
        self.table = torch.empty(4 * n_pairs, dtype=torch.int64, device=dev)
        probe = _lib.MoeCall()
        probe.geom = ctypes.pointer(key[-1])
        probe.n_tokens, probe.top_k, probe.n_experts = 1, n_pairs, n_pairs
        self.scratch = torch.empty(max(_lib.lib().vy_moe_workspace_size(ctypes.byref(probe), PATH_DECODE), 256),
                                   dtype=torch.uint8, device=dev)
        self.sum = torch.empty(x.shape, dtype=torch.float32, device=dev)
        self.cast = torch.empty(x.shape, dtype=x.dtype, device=dev) if tail else None
        self.with_shared = (torch.empty(x.shape, dtype=x.dtype, device=dev)
                            if tail and shared is not None else None)
        self.graph = torch.cuda.CUDAGraph()

    @property
    def result(self):
        if not self.tail:
            return self.sum
        return self.with_shared if self.with_shared is not None else self.cast

    def body(self, x, rw, shared):
        """The recorded work: the layer into `sum`, then the epilogue."""
        _decode_from_table(x, self.n, self.key[-1], self.table, rw, self.sum, workspace=self.scratch)
        if self.tail:
            self.cast.copy_(self.sum)
            if self.with_shared is not None:
                torch.add(self.cast, shared, out=self.with_shared)

    def record(self, x, rw, shared):
        dev = x.device
        side = _CAPTURE_STREAMS.get(dev)
        if side is None:
            side = _CAPTURE_STREAMS[dev] = torch.cuda.Stream(device=dev)
        here = torch.cuda.current_stream(dev)
        side.wait_stream(here)
        gc_on = gc.isenabled()
        gc.disable()        # a collection during the recording could run another graph's teardown
        try:
            with torch.cuda.stream(side), torch.no_grad():
                self.graph.capture_begin(pool=torch.cuda.graph_pool_handle(), capture_error_mode="thread_local")
                try:
                    self.body(x, rw, shared)
                finally:
                    self.graph.capture_end()
        finally:
            if gc_on:
                gc.enable()
        here.wait_stream(side)


def packed_experts_decode_graphed(layer, x, pairs, routing_weights, shared, act_fn, tail):
    """`packed_experts_decode` (and, `tail` True, the forward's epilogue `_tail`) as one CUDA graph
    per MoE layer, or None when this call is not the graph's (the caller then runs eagerly).

    Inputs must keep their addresses from call to call (static tensors); a new address records a
    new graph.  Returns a STATIC tensor that the layer's next call overwrites: the fp32 sum
    [1, hidden] (`tail` False) or the epilogue's result (`tail` True)."""
    if layer in _GRAPH_OFF or not pairs:
        return None
    entries = [b for b, _s in pairs]
    if any("flat" not in b or b.get("geom") is None for b in entries):
        return None
    try:
        _one_geometry(entries, "decode graph")
        _checked(x, pairs, routing_weights, act_fn)
    except NotImplementedError:
        return None
    if not (x.is_contiguous() and routing_weights.is_contiguous()):
        _graph_note("calls with strided activations or routing weights run eagerly")
        return None
    if tail and shared is not None and shared.dtype != x.dtype:
        _graph_note(f"a shared-expert output in {shared.dtype} with {x.dtype} activations runs eagerly")
        return None
    geom_s = _geom_struct(*_blob_key(entries[0]))
    key = (len(pairs), x.data_ptr(), routing_weights.data_ptr(), routing_weights.dtype, x.dtype,
           None if shared is None else shared.data_ptr(), bool(tail), _blob_key(entries[0]), geom_s)
    payload = _pairs_table(pairs)
    g = _GRAPHS.get(layer)
    if g is not None and g.key == key:
        with torch.cuda.device(x.device):
            _stage(payload, x.device, into=g.table)
            g.graph.replay()
        g.replays += 1
        GRAPH_STATS["replays"] += 1
        return g.result
    if g is not None:
        GRAPH_STATS["recorded_unused"] += g.replays == 0
        del _GRAPHS[layer]          # its buffers go before the next recording allocates
        del g
    return _record(layer, key, x, pairs, routing_weights, shared, tail, payload)


def _record(layer, key, x, pairs, rw, shared, tail, payload):
    dev = x.device
    with torch.cuda.device(dev):
        want = None
        if layer not in _GRAPH_VERIFIED or dev not in _KERNELS_READY:
            # the eager launch the first recording is held to (it also sets the kernels'
            # attributes up outside any capture)
            eager = torch.empty(x.shape, dtype=torch.float32, device=dev)
            _launch(x, pairs, rw, eager)
            want = _tail(eager, x.dtype, shared) if tail else eager
            _KERNELS_READY.add(dev)
        try:
            g = _DecodeGraph(key, x, len(pairs), shared, tail)
            g.record(x, rw, shared)
            _stage(payload, dev, into=g.table)
            g.graph.replay()
            got = g.result
            if layer not in _GRAPH_VERIFIED:
                if not torch.equal(got, want):
                    _graph_off(layer, "its first replay does not match the eager launch bit for bit")
                    return want
                _GRAPH_VERIFIED.add(layer)
        except Exception as exc:     # the recording failed: this layer keeps the eager path
            first = str(exc).splitlines()[0][:160] if str(exc) else ""
            _graph_off(layer, f"recording raised {type(exc).__name__}: {first}")
            return want if want is not None else _eager_result(x, pairs, rw, shared, tail)
    _GRAPHS[layer] = g
    GRAPH_STATS["recorded"] += 1
    return got


def _eager_result(x, pairs, rw, shared, tail):
    out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    _launch(x, pairs, rw, out)
    return _tail(out, x.dtype, shared) if tail else out


# ── prefill ──────────────────────────────────────────────────────────────────────────────

def _prefill_unsupported(geom, act_dtype, scale_dtype, w_dtype):
    return _unsupported(geom, act_dtype, scale_dtype, w_dtype)


def _prefill_plan(eidx_cpu):
    """Host view of one call's routing: (order, live, counts) -- row ids sorted by expert id
    (stable), the routed ids ascending, rows per live id.  The kernels build the same plan on the
    device; this is kept for callers that want it on the host."""
    eids = eidx_cpu.reshape(-1)
    order = torch.argsort(eids, stable=True)
    per_expert = torch.bincount(eids)
    live = per_expert.nonzero().reshape(-1)
    return order, live, per_expert[live]


def _prefill_payload(eidx_cpu, blobs):
    """(pinned payload, n_live): int64 [3U] addresses of the routed experts' blobs in ascending
    id order, then the call's expert ids remapped to 0..U-1 (int32; -1 for an id with no entry,
    which the kernels drop, as the per-expert loop skips it)."""
    flat = eidx_cpu.reshape(-1).to(torch.int64)
    live = torch.unique(flat)
    have = torch.tensor([int(e) in blobs for e in live.tolist()], dtype=torch.bool)
    live_have = live[have]
    u = live_have.numel()
    remap = torch.searchsorted(live_have, flat)
    remap = torch.where(remap < u, remap, torch.zeros_like(remap))
    hit = (live_have[remap.clamp(max=max(u - 1, 0))] == flat) if u else torch.zeros_like(flat, dtype=torch.bool)
    ids = torch.where(hit, remap, torch.full_like(remap, -1)).to(torch.int32)
    n = flat.numel()
    vals = torch.empty(3 * u + (n + 1) // 2, dtype=torch.int64)
    vals[:3 * u] = torch.tensor([p for e in live_have.tolist() for p in _blob_ptrs(blobs[e])],
                                dtype=torch.int64)
    tail = vals[3 * u:].view(torch.int32)
    tail[:n] = ids
    return vals, u, [blobs[e] for e in live_have.tolist()]


def _prefill_launch(x, eidx_cpu, routing_weights, blobs, out, plan=None, path=PATH_PREFILL,
                    h_out=None, contrib=None) -> None:
    """The grouped kernels over one call.  No checks: `packed_experts_prefill` gates this."""
    dev = x.device
    n_tok, top_k = eidx_cpu.shape
    vals, u, entries = _prefill_payload(eidx_cpu, blobs)
    geom_s = _geom_struct(*_blob_key(entries[0]))
    tbl = _stage(vals, dev)
    ids = tbl[3 * u:].view(torch.int32)
    if x.stride(-1) != 1:
        x = x.contiguous()
    w = routing_weights
    dense_out = out
    if out is not None and out.stride(-1) != 1:
        dense_out = torch.empty(out.shape, dtype=torch.float32, device=dev)
    c = _make_call(geom_s, x, n_tok, top_k, u, tbl.data_ptr(), ids.data_ptr(), _lib.I32, w,
                   w.stride(0), w.stride(1), None, dense_out, contrib, h_out)
    _enqueue(c, path, dev)
    if dense_out is not out:
        out.copy_(dense_out)


def packed_experts_prefill(x, eidx_cpu, routing_weights, blobs, out, act_fn=None) -> None:
    """A multi-token call's routed-expert sum for one MoE layer, written into `out`.

    x               [tokens, hidden], activation dtype, on a CUDA device (a strided view is fine)
    eidx_cpu        [tokens, top_k] int64 on the CPU: the routed expert ids
    routing_weights [tokens, top_k] on x's device (a strided view is fine)
    blobs           {expert id: `build_expert_blob` blob} for the routed experts; a routed id with
                    no entry contributes nothing (the per-expert loop skips it)
    out             [tokens, hidden] float32, overwritten (a strided view is fine)
    The result is a function of (x, routing, weights) alone: a token's output does not depend on
    the tokens it shares the call with, nor on where the blobs live."""
    dev = _lib.require_cuda(x, routing_weights, out, what="packed_experts_prefill")
    if eidx_cpu.dim() != 2 or routing_weights.shape != eidx_cpu.shape:
        raise ValueError("packed_experts_prefill: eidx and routing weights must be [tokens, top_k]")
    if eidx_cpu.numel() == 0:
        out.zero_()
        return
    live = [int(e) for e in torch.unique(eidx_cpu).tolist() if int(e) in blobs]
    if not live:
        out.zero_()
        return
    entries = [blobs[e] for e in live]
    _one_geometry(entries, "packed_experts_prefill")
    blob = entries[0]
    key = (blob["geom"], x.dtype, routing_weights.dtype, blob["flat"]["scale"].dtype)
    if key not in _PF_VERDICTS:
        _PF_VERDICTS[key] = _prefill_unsupported(blob["geom"], x.dtype,
                                                 blob["flat"]["scale"].dtype, routing_weights.dtype)
    if _PF_VERDICTS[key] is not None:
        raise NotImplementedError(f"fused packed-expert prefill kernels: {_PF_VERDICTS[key]}")
    with torch.cuda.device(dev):
        _prefill_launch(x, eidx_cpu, routing_weights, blobs, out, path=_prefill_path())


def _prefill_path() -> int:
    """Which kernels serve prefill calls: the tcgen05 grouped GEMM when the library has it."""
    return PATH_PREFILL if prefill_available() else PATH_DECODE


@functools.lru_cache(maxsize=None)
def prefill_available() -> bool:
    """True when libvaayu_b200 was built with the tcgen05 grouped-GEMM prefill kernels."""
    return _lib.lib().vy_moe_workspace_size(None, PATH_PREFILL) != 0 or _probe_prefill()


def _probe_prefill() -> bool:
    g = _geom_struct((4, 128, (("gate", 128, 128), ("down", 128, 128), ("up", 128, 128))),
                     torch.bfloat16, False)
    c = _lib.MoeCall()
    c.geom = ctypes.pointer(g)
    c.n_tokens, c.top_k, c.n_experts = 1, 1, 1
    return _lib.lib().vy_moe_workspace_size(ctypes.byref(c), PATH_PREFILL) != 0


# ── device-resident experts (no host sync; graph-capturable) ─────────────────────────────

class ExpertTable:
    """A layer's resident expert blobs as ONE device pointer table [n_experts][3].

    Blobs stay owned by the caller (the table holds references so they outlive it).  Every
    entry must be a blob of one geometry and format."""

    def __init__(self, blobs):
        blobs = list(blobs)
        if not blobs:
            raise ValueError("ExpertTable: no experts")
        _one_geometry(blobs, "ExpertTable")
        self.blobs = blobs
        self.geom = blobs[0]["geom"]
        self.scale_dtype = blobs[0]["flat"]["scale"].dtype
        self.has_zero = "zero" in blobs[0]["flat"]
        self.device = blobs[0]["flat"]["packed"].device
        self.n_experts = len(blobs)
        host = torch.tensor([p for b in blobs for p in _blob_ptrs(b)], dtype=torch.int64)
        self.table = host.to(self.device)
        self.geom_s = _geom_struct(self.geom, self.scale_dtype, self.has_zero)
        lay = blob_layout(self.geom)
        self.hidden, self.inter = lay["gate"][3], lay["gate"][2]

    def weight_bytes(self, experts=None) -> int:
        """HBM bytes of the given experts' streams (all experts by default)."""
        idx = range(self.n_experts) if experts is None else experts
        return sum(t.numel() * t.element_size() for i in idx for t in self.blobs[i]["flat"].values())


FLAG_BAD_EXPERT, FLAG_TIMEOUT, FLAG_DRAIN = 1, 4, 8
_FLAG_TEXT = {FLAG_BAD_EXPERT: "a routed expert's streams were unusable (null or misaligned pointer); "
                               "its slots contributed nothing",
              FLAG_TIMEOUT: "a device-side barrier wait ran out; part of the output is not valid",
              FLAG_DRAIN: "draining in-flight copies after a timeout ran out as well"}


def describe_flags(flags: int) -> str:
    return "; ".join(t for b, t in _FLAG_TEXT.items() if flags & b) or "clean"


def _check_flags(c, path, dev) -> None:
    """Synchronising read of a call's device error flags; raises RuntimeError when any is set."""
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.check(_lib.lib().vy_moe_error_flags(ctypes.byref(c), path, flags.data_ptr(), _lib.stream_of(dev)),
               "vy_moe_error_flags")
    v = int(flags.item())
    if v:
        raise RuntimeError(f"moe_forward: device error flags {v:#x}: {describe_flags(v)}")


def moe_forward(x, expert_ids, routing_weights, table: ExpertTable, out=None, *, path=None,
                contrib=None, h_out=None, w_index=None, workspace=None, expert_base=0, col_blocks=0,
                check=False, shared_last=False, result=None, k_splits=0):
    """The layer over a resident `ExpertTable` with the routing already on the device.

    x [T, hidden] act dtype; expert_ids [T, K] int32/int64 (indices into `table`; an id outside
    it is dropped); routing_weights [T, K] (strided views fine); out [T, hidden] fp32, or
    `contrib` [T*K, hidden] fp32 for the per-row weighted contributions (expert-parallel combine
    on the home rank).  path: PATH_DECODE (token-batched GEMV) or PATH_PREFILL (tcgen05); default
    by call size (prefill above 12 routed rows per expert on average: the B200 crossover measured
    on the cfg1, cfg3 and Mixtral shapes lies between 8 and 16).  expert_base: expert_ids are global ids and the table holds [expert_base,
    expert_base + n) (others drop their slot); expert_ids may be a row-strided view.  col_blocks:
    tokens per decode pass of an expert in blocks of 8 (1, 2, 4; 0 = from the call size).
    k_splits: decode warps sharing one gate/up unit's K range (0 = the library's choice, 1 = none,
    2 / 4 / 8); the result does not depend on it.
    shared_last: slot K - 1 of every token is the block's shared expert (a table entry routed with
    weight 1 or its sigmoid gate); the call then ends with the model's epilogue
    result = act(act(routed fp32 sum) + act(shared contribution)) into `result` [T, hidden] act
    dtype (allocated when None) and returns it, `out` (optional) receiving the routed sum.
    Nothing here synchronises with the host -- except `check=True`, which reads the call's device
    error flags afterwards and raises RuntimeError when any is set."""
    dev = _lib.require_cuda(x, expert_ids, routing_weights, out, contrib, what="moe_forward")
    _check_x(x, "moe_forward")
    key = (table.geom, x.dtype, table.scale_dtype, routing_weights.dtype)
    why = _LAYER_VERDICTS.get(key, False)
    if why is False:                     # first call with this geometry and these dtypes
        why = _LAYER_VERDICTS[key] = _unsupported(*key)
    if why is not None:
        raise NotImplementedError(f"moe_forward: {why}")
    n_tok, top_k = expert_ids.shape
    ids = expert_ids if expert_ids.stride(1) == 1 else expert_ids.contiguous()
    ids_code = _lib.DTYPE_CODE[ids.dtype]
    if shared_last:
        if contrib is not None:
            raise RuntimeError("moe_forward: shared_last needs the layer's own combine (no contrib)")
        if result is None:
            result = torch.empty(n_tok, table.hidden, dtype=x.dtype, device=dev)
        elif result.dtype != x.dtype or result.stride(-1) != 1:
            raise RuntimeError("moe_forward: result must be [T, hidden] in the activation dtype")
    elif out is None and contrib is None:
        out = torch.empty(n_tok, table.hidden, dtype=torch.float32, device=dev)
    if path is None:
        path = PATH_PREFILL if (n_tok * top_k > PREFILL_ROWS_PER_EXPERT * table.n_experts
                                and prefill_available()) else PATH_DECODE
    with torch.cuda.device(dev):
        c = _make_call(table.geom_s, x, n_tok, top_k, table.n_experts, table.table.data_ptr(),
                       ids.data_ptr(), ids_code, routing_weights, routing_weights.stride(0),
                       routing_weights.stride(1), _lib.ptr(w_index), out, contrib, h_out)
        c.expert_base, c.col_blocks, c.k_splits = int(expert_base), int(col_blocks), int(k_splits)
        c.ids_row_stride = ids.stride(0)
        if shared_last:
            c.shared_last = 1
            c.result, c.result_row_stride = result.data_ptr(), (result.stride(0) if result.dim() == 2 else table.hidden)
        _enqueue(c, path, dev, workspace)
        if check:
            _check_flags(c, path, dev)
    return result if shared_last else out


def shared_expert_forward(x, shared: ExpertTable, gate=None, out=None, *, workspace=None):
    """The always-on shared expert of a MoE block on the kernels (`_shared_expert_output`,
    vaayu/moe_patch.py:554-580): `shared` is a one-expert table.  Ungated (DeepSeek): the expert's
    output act(h . Wd) in fp32.  Gated (Qwen2 / Qwen3-Next): `gate` [T] or [T, 1] holds
    sigmoid(gate logits) in the activation dtype, and the product rounds to it as the model's
    `sigmoid(gate(x)) * shared(x)` does.  Returns out [T, hidden] fp32."""
    dev = x.device
    T = x.shape[0]
    ids = torch.zeros(T, 1, dtype=torch.int32, device=dev)
    w = torch.ones(T, 1, dtype=torch.float32, device=dev) if gate is None else gate.reshape(T, 1)
    return moe_forward(x, ids, w, shared, out=out, path=PATH_DECODE, workspace=workspace)


_SHARED_BUFS: dict = {}


def _with_shared(table: ExpertTable, shared: ExpertTable) -> ExpertTable:
    """`table` with `shared`'s expert appended as entry n_experts (cached on the table)."""
    cache = table.__dict__.setdefault("_shared_ext", {})
    hit = cache.get(id(shared))
    if hit is None or hit[0] is not shared:
        hit = (shared, ExpertTable(list(table.blobs) + list(shared.blobs)))
        cache[id(shared)] = hit
    return hit[1]


def _shared_inputs(expert_ids, routing_weights, gate, n_experts):
    """[T, K + 1] ids and weights: the routed slots, then the shared expert (index n_experts,
    weight 1 or the gate) -- reused buffers whose constant column is written once."""
    T, K = expert_ids.shape
    key = (T, K, expert_ids.dtype, routing_weights.dtype, expert_ids.device, n_experts, gate is None)
    bufs = _SHARED_BUFS.get(key)
    if bufs is None:
        ids = torch.full((T, K + 1), n_experts, dtype=expert_ids.dtype, device=expert_ids.device)
        w = torch.ones(T, K + 1, dtype=routing_weights.dtype, device=routing_weights.device)
        bufs = _SHARED_BUFS[key] = (ids, w)
    ids, w = bufs
    ids[:, :K].copy_(expert_ids)
    w[:, :K].copy_(routing_weights)
    if gate is not None:
        w[:, K].copy_(gate.reshape(T))
    return ids, w


def moe_forward_with_shared(x, expert_ids, routing_weights, table: ExpertTable, shared: ExpertTable,
                            gate=None, out=None, *, fused=True, result=None, **kw):
    """The routed layer plus the shared expert, combined as the reference's epilogue does
    (`_tail`, vaayu/packed_expert_kernels.py:502-508): out.to(act) + shared.to(act).  Returns the
    act-dtype result; `out` (optional) receives the routed fp32 sum.

    fused (default): ONE layer call -- the shared expert is appended to the table as an always-
    routed extra slot of every token (weight 1, or the gate in the routing weights' dtype) and the
    layer's combine applies the epilogue; bit-identical to the two-call form.  It is taken when the
    shared expert has the routed experts' geometry and format, the gate converts exactly to the
    routing-weight dtype, and no expert_base / contrib / w_index is given; otherwise the shared
    expert runs as its own call (`shared_expert_forward`)."""
    exact_gate = gate is None or routing_weights.dtype in (torch.float32, gate.dtype)
    if (fused and exact_gate and shared.n_experts == 1 and shared.geom == table.geom
            and shared.scale_dtype == table.scale_dtype and shared.has_zero == table.has_zero
            and not kw.get("expert_base") and kw.get("contrib") is None and kw.get("w_index") is None):
        ids, w = _shared_inputs(expert_ids, routing_weights, gate, table.n_experts)
        return moe_forward(x, ids, w, _with_shared(table, shared), out=out, shared_last=True, result=result, **kw)
    out = moe_forward(x, expert_ids, routing_weights, table, out=out, **kw)
    res = _tail(out, x.dtype, shared_expert_forward(x, shared, gate))
    if result is not None:
        result.copy_(res)
        return result
    return res


def moe_workspace_bytes(table: ExpertTable, n_tokens: int, top_k: int, path: int = PATH_DECODE,
                        contrib: bool = False, col_blocks: int = 0, k_splits: int = 0) -> int:
    """Scratch bytes one `moe_forward` call of this size needs (to preallocate for graphs)."""
    c = _lib.MoeCall()
    c.geom = ctypes.pointer(table.geom_s)
    c.n_tokens, c.top_k, c.n_experts = n_tokens, top_k, table.n_experts
    c.contrib = 1 if contrib else None
    c.col_blocks, c.k_splits = int(col_blocks), int(k_splits)
    return int(_lib.lib().vy_moe_workspace_size(ctypes.byref(c), path))


def combine(contrib, expert_ids, out=None):
    """out[t] = token t's rows of `contrib` [T*K, hidden] summed in ascending expert id, then
    slot (fp32) -- the expert-parallel combine on the token's home rank."""
    dev = _lib.require_cuda(contrib, expert_ids, out, what="combine")
    n_tok, top_k = expert_ids.shape
    hidden = contrib.shape[-1]
    ids = expert_ids.contiguous()
    if out is None:
        out = torch.empty(n_tok, hidden, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().vy_moe_combine(
            contrib.contiguous().data_ptr(), ids.data_ptr(), _lib.DTYPE_CODE[ids.dtype], n_tok,
            top_k, hidden, out.data_ptr(), out.stride(0), _lib.stream_of(dev)), "combine")
    return out


# ── install into a Vaayu engine ──────────────────────────────────────────────────────────
#
# The engine calls `install_packed_expert_kernels(self)` once at load; it routes the blocks
# whose forward is the fused sparse one.  Decision, in order: a CUDA model on the current device,
# the library present, SiLU experts, one real expert of the first fused block readable as a blob
# whose geometry and dtypes the kernels take (decode, for every fused block); then prefill for
# each block whose own first expert has the same format and whose expert set fits a quarter of
# the device's free memory at install time (a prefill call holds every routed expert at once).

_FUSED_FORWARD = "_make_fused_sparse_forward"    # the engine's name for the fused MoE forward


def _is_silu(act_fn, device, dtype) -> bool:
    """Does the experts' activation compute SiLU on this dtype? (the kernels hardcode it)"""
    if act_fn is None:
        return False
    probe = torch.linspace(-12.0, 12.0, 301, device=device).to(dtype)
    try:
        return torch.equal(act_fn(probe), torch.nn.functional.silu(probe))
    except Exception:
        return False


def _layer_file_blob(checkpoint_path, layer_name, device):
    """The blob of the lowest-numbered expert stored in `<checkpoint_path>/<layer_name>.safetensors`,
    read with this package's checkpoint reader (that expert's tensors only), or None."""
    from .checkpoint import Checkpoint
    path = os.path.join(str(checkpoint_path), f"{layer_name}.safetensors")
    if not os.path.isfile(path):
        return None
    ck = Checkpoint(path)
    try:
        found = ck.lowest_expert()
        return None if found is None else ck.expert_blob(found[0], found[1], device)
    finally:
        ck.close()


def _probe_blob(vaayu_ref, block, device):
    """One real expert of `block` as a blob: the host's own `packed_probe_blob(block, device)` when
    it has one, else the block's layer file under `checkpoint_path`.  NotImplementedError from
    `build_expert_blob` (act-order, mixed widths) propagates."""
    probe = getattr(vaayu_ref, "packed_probe_blob", None)
    if callable(probe):
        return probe(block, device)
    ckpt, name = getattr(vaayu_ref, "checkpoint_path", None), getattr(block, "layer_name", None)
    if ckpt is None or name is None:
        return None
    return _layer_file_blob(ckpt, name, device)


def _format_of(blob):
    return blob["geom"], blob["flat"]["scale"].dtype, "zero" in blob["flat"]


def _install_refusal(vaayu_ref, device, dtype, block):
    """Why the kernels cannot serve this model at all, or None."""
    current = torch.cuda.current_device()
    if device.index is not None and device.index != current:
        return (f"the model runs on {device}, not the current CUDA device cuda:{current} "
                "(the kernels launch on the current device)")
    act_fn = getattr(getattr(block.moe_module, block.experts_attr, None), "act_fn", None)
    if not _is_silu(act_fn, device, dtype):
        return "the experts' activation is not SiLU"
    return None


def install_packed_expert_kernels(vaayu_ref) -> bool:
    """Serve the engine's fused pack-quantized MoE blocks with these kernels: one-token decode of
    every such block, and prefill of each block whose experts share the first block's format.
    Sets `vaayu_ref._packed_moe_kernel` (the geometry served) and, when any block qualifies,
    `vaayu_ref._packed_moe_prefill_kernel` (frozenset of their `layer_idx`).  Returns whether the
    decode kernels were installed; when they are not, the reason is logged and the engine keeps
    its own path."""
    device = torch.device(str(vaayu_ref.running_device))
    if device.type != "cuda" or not _lib.LIB_PATH.exists():
        return False
    blocks = [b for b in (getattr(vaayu_ref, "_moe_blocks", None) or [])
              if getattr(b, "forward_name", None) == _FUSED_FORWARD]
    if not blocks:
        return False
    dtype, first = vaayu_ref.running_dtype, blocks[0]
    why, blob = _install_refusal(vaayu_ref, device, dtype, first), None
    if why is None:
        try:
            blob = _probe_blob(vaayu_ref, first, device)
        except NotImplementedError as exc:
            why = str(exc)
        if blob is None and why is None:
            why = f"no pack-quantized expert of layer {first.layer_idx} could be read as a blob"
    if why is None:
        why = next((w for w in (_unsupported(blob["geom"], dtype, blob["flat"]["scale"].dtype, rw_dtype)
                                for rw_dtype in (torch.float32, dtype)) if w), None)
    if why is not None:
        log.warning("vaayu_b200: fused expert kernels not installed: %s; the engine keeps its own path", why)
        return False
    vaayu_ref._packed_moe_kernel = blob["geom"]
    bits, gs, _roles = blob["geom"]
    log.info("vaayu_b200: fused int%d expert decode (group %d) on %d MoE layers", bits, gs, len(blocks))

    fmt, blob_bytes = _format_of(blob), sum(t.numel() * t.element_size() for t in blob["flat"].values())
    budget = torch.cuda.mem_get_info(device)[0] // 4
    eligible, left_out = [], collections.defaultdict(list)
    for b in blocks:
        try:
            one = blob if b is first else _probe_blob(vaayu_ref, b, device)
            reason = "no pack-quantized expert could be read as a blob"
        except NotImplementedError as exc:
            one, reason = None, str(exc)
        if one is not None:
            n_exp = int(getattr(getattr(b.moe_module, b.experts_attr, None), "num_experts", 0) or 0)
            if _format_of(one) != fmt:
                reason = "its experts differ in geometry or format from layer %d's" % first.layer_idx
            elif n_exp and n_exp * blob_bytes > budget:
                reason = (f"its {n_exp} experts ({n_exp * blob_bytes / 2**30:.2f} GiB) exceed a quarter "
                          f"of the free device memory at install ({budget / 2**30:.2f} GiB)")
            else:
                eligible.append(b.layer_idx)
                continue
        left_out[reason].append(b.layer_idx)
    if eligible:
        vaayu_ref._packed_moe_prefill_kernel = frozenset(eligible)
        log.info("vaayu_b200: fused int%d expert prefill on %d of %d MoE layers", bits, len(eligible), len(blocks))
    for reason, idxs in left_out.items():
        log.warning("vaayu_b200: prefill of layers %s stays on the engine's path: %s",
                    ", ".join(map(str, idxs)), reason)
    return True
