"""Reading compressed-tensors `pack-quantized` MoE checkpoints into expert blobs.

The on-disk side of the expert layer: int4/int8 GPTQ/AWQ checkpoints store each expert linear as
bit-packed int32 codes + per-group scales (+ zero points), `weight_packed` / `weight_scale` /
`weight_shape` / `weight_zero_point` / `weight_g_idx`.  This module

  - groups one expert's tensors by role exactly as the reference does
    (`_EXPERT_WEIGHT_ROLES` vaayu/moe_patch.py:34-43, `_group_packed_tensors_by_weight` :532-551,
    `_packed_roles_complete` :591-594): a key belongs to the first role whose pattern it contains,
    its component is the text after the last dot;
  - reads only the requested experts' tensors from safetensors files, through a memory map, at the
    checkpoint's own bit width (the reference's sparse read, `load_expert_sparse`,
    vaayu/persist/safetensor_model_persister.py:967) -- nothing is dequantised on the host;
  - builds the kernels' blobs (`build_expert_blob`) and a layer's resident `ExpertTable`.

The safetensors container is parsed here (8-byte little-endian header length, a JSON header of
{name: {dtype, shape, data_offsets}}, then the data), so no extra package is needed.
"""
from __future__ import annotations

import json
import mmap
import os
import re
from typing import Iterable, Optional

import numpy as np
import torch

EXPERT_WEIGHT_ROLES: list[tuple[str, str]] = [
    (".w1.", "gate"), (".w2.", "down"), (".w3.", "up"),                        # Mixtral
    (".gate_proj.", "gate"), (".down_proj.", "down"), (".up_proj.", "up"),     # DeepSeek, Qwen, ...
]
PACKED_COMPONENT_KEYS = {"weight_packed", "weight_scale", "weight_shape", "weight_zero_point",
                         "weight_g_idx"}


def group_packed_tensors_by_weight(raw: dict) -> dict:
    """{"gate": {component: tensor}, "down": ..., "up": ...}; empty dicts for a dense expert."""
    result = {"gate": {}, "down": {}, "up": {}}
    for key, tensor in raw.items():
        role = next((r for pattern, r in EXPERT_WEIGHT_ROLES if pattern in key), None)
        if role is None:
            continue
        component = key.rsplit(".", 1)[-1]
        if component in PACKED_COMPONENT_KEYS:
            result[role][component] = tensor
    return result


def packed_roles_complete(packed: dict) -> bool:
    """Every role has its codes and scales."""
    return all("weight_packed" in packed[r] and "weight_scale" in packed[r] for r in ("gate", "down", "up"))


# ── safetensors ──────────────────────────────────────────────────────────────────────────

_ST_DTYPES = {
    "F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
    "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
    "BOOL": torch.bool, "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2,
}


class SafetensorsFile:
    """One .safetensors file, memory-mapped; `tensor(name)` copies that tensor's bytes only."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        n = int.from_bytes(self._mm[:8], "little")
        if n <= 0 or 8 + n > len(self._mm):
            raise ValueError(f"{path}: not a safetensors file (header length {n})")
        header = json.loads(self._mm[8:8 + n].decode("utf-8"))
        header.pop("__metadata__", None)
        self._data = 8 + n
        self.entries = header

    def keys(self):
        return self.entries.keys()

    def tensor(self, name: str) -> torch.Tensor:
        e = self.entries[name]
        dtype = _ST_DTYPES.get(e["dtype"])
        if dtype is None:
            raise NotImplementedError(f"{self.path}: {name}: safetensors dtype {e['dtype']}")
        lo, hi = e["data_offsets"]
        raw = np.frombuffer(self._mm, dtype=np.uint8, count=hi - lo, offset=self._data + lo).copy()
        return torch.from_numpy(raw).view(dtype).reshape(e["shape"])

    def close(self):
        self._mm.close()
        self._f.close()


class Checkpoint:
    """The tensors of one or more safetensors files by name (the files of a sharded checkpoint)."""

    def __init__(self, paths: "str | Iterable[str]"):
        if isinstance(paths, (str, os.PathLike)):
            p = str(paths)
            paths = sorted(os.path.join(p, f) for f in os.listdir(p) if f.endswith(".safetensors")) \
                if os.path.isdir(p) else [p]
        self.files = [SafetensorsFile(p) for p in paths]
        self.index = {k: f for f in self.files for k in f.keys()}

    def close(self):
        for f in self.files:
            f.close()

    def expert_keys(self, layer_prefix: str, expert: int) -> list:
        """Keys of expert `expert` under `layer_prefix` (e.g. "model.layers.3.mlp")."""
        head = f"{layer_prefix}.experts.{expert}."
        return [k for k in self.index if k.startswith(head)]

    def experts(self, layer_prefix: str) -> list:
        """Expert ids present under `layer_prefix`, ascending."""
        pat = re.compile(re.escape(layer_prefix) + r"\.experts\.(\d+)\.")
        return sorted({int(m.group(1)) for k in self.index for m in [pat.match(k)] if m})

    def lowest_expert(self):
        """(layer prefix, expert id) of the lowest-numbered expert stored anywhere in these files
        (keys "<prefix>.experts.<id>.<...>"), or None when they hold no expert tensors."""
        pat = re.compile(r"^(.*)\.experts\.(\d+)\.")
        found = [(int(m.group(2)), m.group(1)) for k in self.index for m in [pat.match(k)] if m]
        if not found:
            return None
        e, prefix = min(found)
        return prefix, e

    def read_expert(self, layer_prefix: str, expert: int) -> dict:
        """{key: tensor} of one expert: the sparse read (only its own bytes)."""
        return {k: self.index[k].tensor(k) for k in self.expert_keys(layer_prefix, expert)}

    def expert_blob(self, layer_prefix: str, expert: int, device="cuda") -> Optional[dict]:
        """The kernels' blob of one pack-quantized expert (None when it is dense or incomplete)."""
        from .moe_patch import build_expert_blob
        packed = group_packed_tensors_by_weight(self.read_expert(layer_prefix, expert))
        if not packed["gate"] or not packed_roles_complete(packed):
            return None
        on_dev = {r: {k: (v if k == "weight_shape" else v.to(device)) for k, v in packed[r].items()}
                  for r in ("gate", "down", "up")}
        return build_expert_blob(on_dev)

    def layer_table(self, layer_prefix: str, experts: "Iterable[int] | None" = None, device="cuda"):
        """A resident `ExpertTable` of the layer's experts (all, or the given ascending range --
        one expert-parallel rank's share)."""
        from .packed_expert_kernels import ExpertTable
        ids = list(experts) if experts is not None else self.experts(layer_prefix)
        blobs = []
        for e in ids:
            b = self.expert_blob(layer_prefix, e, device)
            if b is None:
                raise NotImplementedError(f"{layer_prefix}.experts.{e} is not a complete pack-quantized expert")
            blobs.append(b)
        return ExpertTable(blobs)


def write_safetensors(path: str, tensors: dict, metadata: Optional[dict] = None) -> None:
    """Write `tensors` ({name: tensor}) as a safetensors file (for tests and tooling)."""
    names = sorted(tensors)
    rev = {v: k for k, v in _ST_DTYPES.items()}
    header, offset, blobs = {}, 0, []
    for n in names:
        t = tensors[n].detach().contiguous().cpu()
        b = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[n] = {"dtype": rev[t.dtype], "shape": list(t.shape), "data_offsets": [offset, offset + len(b)]}
        offset += len(b)
        blobs.append(b)
    if metadata:
        header["__metadata__"] = metadata
    hj = json.dumps(header).encode("utf-8")
    hj += b" " * ((-len(hj)) % 8)
    with open(path, "wb") as f:
        f.write(len(hj).to_bytes(8, "little"))
        f.write(hj)
        for b in blobs:
            f.write(b)
