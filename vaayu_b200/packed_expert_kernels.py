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
    False with a WARNING for a model it cannot serve, leaving the engine's own path in place.
  * The verdict is a geometry gate only (`_unsupported`); the first-call comparison against the
    stock arithmetic lives in the test suite, not in the product.
  * Zero-point blobs are served (see vaayu_b200.moe_patch).
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
    """Why the kernels cannot run a call with this geometry and these dtypes, or None."""
    bits, gs, roles = geom
    shapes = {r: (rows, cols) for r, rows, cols in roles}
    if set(shapes) != set(_ROLES):
        return f"expert roles {sorted(shapes)} are not gate/up/down"
    inter, hid = shapes["gate"]
    if shapes["up"] != (inter, hid) or shapes["down"] != (hid, inter):
        return f"projection shapes {shapes} are not a gated MLP"
    if bits != 4:
        return f"{bits}-bit codes (the expert kernels take int4)"
    if gs & (gs - 1) or gs < 32:
        return f"group size {gs} is not a power of two >= 32"
    if hid % 128 or inter % 128 or hid % gs or inter % gs:
        return (f"hidden {hid} / intermediate {inter} are not multiples of 128 and of the "
                f"group size {gs}")
    if act_dtype not in (torch.bfloat16, torch.float16):
        return f"activation dtype {act_dtype} (bf16 / fp16)"
    for what, dt in (("scale", scale_dtype), ("routing-weight", w_dtype)):
        if dt not in _DTYPE_CODE:
            return f"{what} dtype {dt}"
    return None


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


# ── per-stream scratch and the pinned table ring ─────────────────────────────────────────

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


class _TableRing:
    """Pinned staging for a call's table, reused round-robin.  A slot's host buffer is rewritten
    only after the H2D copy that last read it completed (its event); each slot has its own device
    buffer, so no queued kernel's table is overwritten (vaayu/packed_expert_kernels.py:263-292)."""

    def __init__(self, n_slots: int = 4):
        self._slots: list = [None] * n_slots
        self._next = 0

    def put(self, values: torch.Tensor, device) -> torch.Tensor:
        i = self._next
        self._next = (i + 1) % len(self._slots)
        n = values.numel()
        slot = self._slots[i]
        if slot is None or slot[0].numel() < n or slot[1].device != device:
            host = torch.empty(max(64, 1 << (n - 1).bit_length()), dtype=torch.int64, pin_memory=True)
            slot = self._slots[i] = [host, torch.empty(host.shape, dtype=torch.int64, device=device),
                                     torch.cuda.Event(), False]
        host, dev, done, used = slot
        if used:
            done.synchronize()
        host[:n] = values
        dev[:n].copy_(host[:n], non_blocking=True)
        done.record()
        slot[3] = True
        return dev


_TABLES = _TableRing()
_PF_TABLES = _TableRing()
_VERDICTS: dict = {}
_PF_VERDICTS: dict = {}


# ── the call itself ──────────────────────────────────────────────────────────────────────

def _make_call(geom_s, x, n_tokens, top_k, n_experts, table_ptr, ids_ptr, ids_code, rw,
               w_tok_stride, w_slot_stride, w_index_ptr, out, contrib, h_out) -> _lib.MoeCall:
    c = _lib.MoeCall()
    c.geom = ctypes.pointer(geom_s)
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
    """Pinned-ring payload of a decode call: int64 [4n] = n x (packed, scale, zero) addresses,
    then n int32 expert indices (0..n-1, the table order) and n int32 slots."""
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
    blob0 = pairs[0][0]
    geom_s = _geom_struct(*_blob_key(blob0))
    tbl = _TABLES.put(_pairs_table(pairs), x.device)
    _decode_from_table(x, len(pairs), geom_s, tbl, routing_weights, out, h_out)


def _checked(x, pairs, routing_weights, act_fn=None) -> None:
    """The cached geometry verdict for this call's (geometry, dtypes) key; raises when the
    kernels cannot take it."""
    blob = pairs[0][0]
    key = (blob["geom"], x.dtype, routing_weights.dtype, blob["flat"]["scale"].dtype)
    if key not in _VERDICTS:
        _VERDICTS[key] = _unsupported(blob["geom"], x.dtype, blob["flat"]["scale"].dtype,
                                      routing_weights.dtype)
    why = _VERDICTS[key]
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


# ── one CUDA graph per MoE layer (vaayu/packed_expert_kernels.py:483-654) ────────────────────

_GRAPHS: dict = {}              # layer -> _LayerGraph
_GRAPH_REFUSED: dict = {}       # layer -> why
_GRAPH_WARNED: set = set()
_GRAPH_STREAMS: dict = {}       # device -> capture stream
GRAPH_STATS: collections.Counter = collections.Counter()


class _LayerGraph:
    __slots__ = ("key", "graph", "host", "tbl", "ws", "out", "tmp", "result", "done", "replays")


def _tail(out, dtype, shared):
    """The forward's epilogue: the fp32 sum cast back, plus the shared expert's output."""
    result = out.to(dtype)
    if shared is not None:
        result = result + shared.to(result.dtype)
    return result


def _refuse_graph(layer, why) -> None:
    _GRAPH_REFUSED[layer] = why
    _GRAPHS.pop(layer, None)
    GRAPH_STATS["refused"] += 1
    if why not in _GRAPH_WARNED:
        _GRAPH_WARNED.add(why)
        print(f"[Vaayu] WARNING: packed-expert decode graph refused for MoE layer {layer} "
              f"({why}); it launches eagerly. Later layers refused for the same reason are "
              f"not listed.")


def _warn_skip(why) -> None:
    if why not in _GRAPH_WARNED:
        _GRAPH_WARNED.add(why)
        print(f"[Vaayu] WARNING: packed-expert decode graph not used ({why}); those calls "
              f"launch the kernels eagerly. Shown once per reason.")


def packed_experts_decode_graphed(layer, x, pairs, routing_weights, shared, act_fn, tail):
    """`packed_experts_decode` (and, `tail` True, the forward's epilogue) through one CUDA graph
    per MoE layer -- or None: this call is not the graph's, run the eager path.

    The caller passes only inputs whose addresses hold from call to call.  Returns a STATIC
    tensor the layer's next call overwrites: the fp32 sum [1, hidden] (`tail` False) or
    `_tail(sum, x.dtype, shared)` (`tail` True)."""
    if layer in _GRAPH_REFUSED:
        return None
    blob0 = pairs[0][0]
    geom = blob0.get("geom")
    if geom is None or "flat" not in blob0 or any(
            blob.get("geom") != geom or "flat" not in blob for blob, _slot in pairs[1:]):
        return None
    if not (x.is_contiguous() and routing_weights.is_contiguous()):
        _warn_skip("a non-contiguous expert input or routing-weight tensor")
        return None
    if tail and shared is not None and shared.dtype != x.dtype:
        _warn_skip(f"the shared expert's output is {shared.dtype}, the activations {x.dtype}")
        return None
    try:
        _one_geometry([b for b, _s in pairs], "packed_experts_decode_graphed")
        _checked(x, pairs, routing_weights, act_fn)
    except NotImplementedError:
        return None
    vals = _pairs_table(pairs)
    key = (len(pairs), x.data_ptr(), routing_weights.data_ptr(), routing_weights.dtype,
           0 if shared is None else shared.data_ptr(), tail, geom, x.dtype,
           blob0["flat"]["scale"].dtype, "zero" in blob0["flat"])
    g = _GRAPHS.get(layer)
    if g is not None and g.key == key:
        g.done.synchronize()            # this layer's last replay has read the table
        g.host.copy_(vals)
        g.graph.replay()
        g.done.record()
        g.replays += 1
        GRAPH_STATS["replays"] += 1
        return g.result if tail else g.out
    if g is not None:
        del _GRAPHS[layer]
        if g.replays == 0:
            GRAPH_STATS["replaced_unreplayed"] += 1
        del g
    return _capture(layer, key, x, pairs, routing_weights, shared, tail, vals)


def _capture(layer, key, x, pairs, rw, shared, tail, vals):
    dev = x.device
    n = len(pairs)
    geom_s = _geom_struct(*_blob_key(pairs[0][0]))
    with torch.cuda.device(dev):
        ref_out = torch.empty(x.shape, dtype=torch.float32, device=dev)
        _launch(x, pairs, rw, ref_out)
        ref = _tail(ref_out, x.dtype, shared) if tail else ref_out
        g = _LayerGraph()
        graph = torch.cuda.CUDAGraph()
        pool = torch.cuda.graph_pool_handle()
        was = gc.isenabled()
        gc.disable()
        try:
            g.key, g.replays = key, 0
            g.host = torch.empty(len(vals), dtype=torch.int64, pin_memory=True)
            g.host.copy_(vals)
            g.tbl = torch.empty(len(vals), dtype=torch.int64, device=dev)
            c_probe = _lib.MoeCall()
            c_probe.geom = ctypes.pointer(geom_s)
            c_probe.n_tokens, c_probe.top_k, c_probe.n_experts = 1, n, n
            need = _lib.lib().vy_moe_workspace_size(ctypes.byref(c_probe), PATH_DECODE)
            g.ws = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
            g.out = torch.empty(x.shape, dtype=torch.float32, device=dev)
            g.tmp = torch.empty(x.shape, dtype=x.dtype, device=dev) if tail else None
            g.result = (torch.empty(x.shape, dtype=x.dtype, device=dev)
                        if tail and shared is not None else g.tmp)
            g.done = torch.cuda.Event()
            side = _GRAPH_STREAMS.get(dev)
            if side is None:
                side = _GRAPH_STREAMS[dev] = torch.cuda.Stream(device=dev)
            cur = torch.cuda.current_stream(dev)
            side.wait_stream(cur)
            with torch.cuda.stream(side), torch.no_grad():
                graph.capture_begin(pool=pool, capture_error_mode="thread_local")
                try:
                    g.tbl.copy_(g.host, non_blocking=True)
                    _decode_from_table(x, n, geom_s, g.tbl, rw, g.out, workspace=g.ws)
                    if tail:
                        g.tmp.copy_(g.out)
                        if shared is not None:
                            torch.add(g.tmp, shared, out=g.result)
                finally:
                    graph.capture_end()
            cur.wait_stream(side)
            g.graph = graph
            graph.replay()
            got = g.result if tail else g.out
            same = torch.equal(got, ref)
        except Exception as exc:
            first = (str(exc).splitlines() or [""])[0][:200]
            _refuse_graph(layer, f"capture failed: {type(exc).__name__}: {first}")
            return ref
        finally:
            if was:
                gc.enable()
        if not same:
            _refuse_graph(layer, "its replay disagrees bitwise with the eager launch")
            return ref
        g.done.record()
        _GRAPHS[layer] = g
        GRAPH_STATS["captures"] += 1
        return got


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
    tbl = _PF_TABLES.put(vals, dev)
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
    why = _unsupported(table.geom, x.dtype, table.scale_dtype, routing_weights.dtype)
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


# ── install (vaayu/packed_expert_kernels.py:864-1012) ────────────────────────────────────────

def _is_silu(act_fn, device, dtype) -> bool:
    """Behavioural: does the experts' activation compute SiLU? (the kernels hardcode it)"""
    if act_fn is None:
        return False
    t = torch.linspace(-8.0, 8.0, 257, device=device).to(dtype)
    try:
        return torch.equal(act_fn(t), torch.nn.functional.silu(t))
    except Exception:
        return False


def _one_real_blob(vaayu_ref, block, device, quiet=False):
    """The blob of `block`'s lowest-numbered expert.  Inside Vaayu the engine's own loader
    reads it off the checkpoint; any other host supplies `vaayu_ref.packed_probe_blob(block,
    device)`."""
    probe = getattr(vaayu_ref, "packed_probe_blob", None)
    why = "its projections are packed at different bit widths or group sizes"
    try:
        if callable(probe):
            blob = probe(block, device)
        else:
            from vaayu.moe_patch import (_group_packed_tensors_by_weight, _packed_roles_complete,
                                         _upload_packed_expert)
            from vaayu.persist.safetensor_model_persister import load_expert_sparse
            from pathlib import Path
            from .moe_patch import build_expert_blob
            metas = vaayu_ref._expert_offset_index.index.get(block.layer_name, {})
            if not metas:
                return None
            raw = load_expert_sparse(str(Path(vaayu_ref.checkpoint_path) / f"{block.layer_name}.safetensors"),
                                     metas[min(metas)])
            packed = _group_packed_tensors_by_weight(raw)
            if not packed["gate"] or not _packed_roles_complete(packed):
                return None
            blob = build_expert_blob(_upload_packed_expert(packed, device))
    except NotImplementedError as exc:
        blob, why = None, str(exc)
    if blob is None and not quiet:
        print(f"[Vaayu] WARNING: fused packed-expert decode kernel not installed: {why}")
    return blob


def install_packed_expert_kernels(vaayu_ref) -> bool:
    """Route the fused pack-quantized MoE blocks through the kernels -- one-token decode of every
    such block, and the prefill calls of each block whose geometry matches -- if the kernels can
    take this model's geometry on this device.  Sets `vaayu_ref._packed_moe_kernel` (the
    geometry) and `vaayu_ref._packed_moe_prefill_kernel` (frozenset of eligible `layer_idx`).
    Returns whether the decode kernel was installed; a refusal is reported with a WARNING and
    leaves the engine's own path in place."""
    device = str(vaayu_ref.running_device)
    if torch.device(device).type != "cuda" or not _lib.LIB_PATH.exists():
        return False
    blocks = [b for b in (getattr(vaayu_ref, "_moe_blocks", None) or [])
              if getattr(b, "forward_name", None) == "_make_fused_sparse_forward"]
    if not blocks:
        return False
    dev_index = torch.device(device).index
    if dev_index is not None and dev_index != torch.cuda.current_device():
        print(f"[Vaayu] WARNING: fused packed-expert decode kernel not installed: model "
              f"device {device} is not the current CUDA device "
              f"({torch.cuda.current_device()}); decode keeps the stock per-expert path")
        return False
    block, dtype = blocks[0], vaayu_ref.running_dtype
    act_fn = getattr(getattr(block.moe_module, block.experts_attr, None), "act_fn", None)
    if not _is_silu(act_fn, device, dtype):
        print("[Vaayu] fused packed-expert decode kernel not used: the experts' activation "
              "is not SiLU")
        return False
    blob = _one_real_blob(vaayu_ref, block, device)
    if blob is None:
        return False
    scale_dtype = blob["flat"]["scale"].dtype
    bad = [why for why in (_unsupported(blob["geom"], dtype, scale_dtype, w)
                           for w in (torch.float32, dtype)) if why]
    if bad:
        print(f"[Vaayu] WARNING: fused packed-expert decode kernel refused ({bad[0]}); these "
              f"experts stay on the stock per-expert path")
        return False
    vaayu_ref._packed_moe_kernel = blob["geom"]
    bits, gs, _roles = blob["geom"]
    print(f"[Vaayu] fused packed-expert decode kernel on {len(blocks)} MoE layers "
          f"({bits}-bit, group {gs})")
    checked = (blob["geom"], scale_dtype, "zero" in blob["flat"])
    eligible, skipped = [], {}
    for b in blocks:
        one = blob if b is block else _one_real_blob(vaayu_ref, b, device, quiet=True)
        if one is None:
            why = "experts not pack-quantized, or packed with no fused pass"
        elif (one["geom"], one["flat"]["scale"].dtype, "zero" in one["flat"]) != checked:
            why = "a different geometry or scale dtype than the checked layer"
        else:
            eligible.append(b.layer_idx)
            continue
        skipped.setdefault(why, []).append(b.layer_idx)
    if not eligible:
        print(f"[Vaayu] WARNING: fused packed-expert prefill kernel not installed: "
              f"{'; '.join(skipped)}; prefill keeps the per-expert path")
        return True
    vaayu_ref._packed_moe_prefill_kernel = frozenset(eligible)
    print(f"[Vaayu] fused packed-expert prefill kernel on {len(eligible)} MoE layers "
          f"({bits}-bit, group {gs})")
    if skipped:
        left_out = sorted(i for idxs in skipped.values() for i in idxs)
        print(f"[Vaayu] WARNING: fused packed-expert prefill kernel not used on "
              f"{len(left_out)} of {len(blocks)} MoE layers (layer indices "
              f"{', '.join(map(str, left_out))}): {'; '.join(skipped)}; prefill keeps the "
              f"per-expert path there")
    return True
