"""Cluster-packed expert weights (``.ctsr``): one sequential read into pinned memory.

Mirrors ``chronos/io/storage.py`` of FonaTech/Project_Chronos (``ClusterStorage``,
``ClusterManifest``, ``MANIFEST_FILENAME``; same file layout, key scheme
``l{layer}_e{expert}__{param}`` and manifest JSON), so caches written by either
side read on the other.  A ``.ctsr`` file is a safetensors container: an
8-byte little-endian header length, a JSON header mapping each key to
``dtype`` / ``shape`` / ``data_offsets`` (relative to the data section), then
the raw tensor bytes.

The read path is built for the H2D promotion that follows it: the whole
cluster file is read with one sequential ``readinto`` into ONE page-locked
host buffer, and every tensor is a zero-copy view of that buffer.  A promotion
is then a plain ``cudaMemcpyAsync`` from pinned memory, with no per-tensor
decode or copy on the host (the reference materialises each tensor through
``safe_open.get_tensor``).  The writer produces the same format with no
dependency on the ``safetensors`` package.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch

MANIFEST_FILENAME = "cluster_manifest.json"
MANIFEST_VERSION = 1
KEY_SEP = "__"

# safetensors dtype names <-> torch
_ST_DTYPES = {"F16": torch.float16, "BF16": torch.bfloat16, "F32": torch.float32, "F64": torch.float64,
              "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
              "BOOL": torch.bool}
_ST_NAMES = {v: k for k, v in _ST_DTYPES.items()}


def _key(layer_id: int, expert_id: int, param_name: str) -> str:
    return f"l{layer_id}_e{expert_id}{KEY_SEP}{param_name}"


def _parse_key(key: str) -> Optional[Tuple[int, int, str]]:
    if KEY_SEP not in key:
        return None
    prefix, param = key.split(KEY_SEP, 1)
    if not (prefix.startswith("l") and "_e" in prefix):
        return None
    try:
        layer_s, expert_s = prefix[1:].split("_e", 1)
        return int(layer_s), int(expert_s), param
    except ValueError:
        return None


@dataclass
class ClusterManifest:
    """Parsed ``cluster_manifest.json`` (``chronos/io/storage.py:61-110``)."""
    version: int
    num_experts: int
    num_layers: int
    storage_format: str
    clusters: Dict[int, Tuple[str, List[int]]]   # cluster id -> (file, expert ids)
    expert_to_cluster: Dict[int, int]

    @classmethod
    def from_dict(cls, data: Dict) -> "ClusterManifest":
        clusters = {int(c["cluster_id"]): (c["file"], [int(e) for e in c["experts"]]) for c in data["clusters"]}
        return cls(version=int(data.get("version", MANIFEST_VERSION)), num_experts=int(data["num_experts"]),
                   num_layers=int(data["num_layers"]),
                   storage_format=data.get("storage_format", "safetensors"), clusters=clusters,
                   expert_to_cluster={int(k): int(v) for k, v in data["expert_to_cluster"].items()})

    def to_dict(self) -> Dict:
        return {"version": self.version, "num_experts": self.num_experts, "num_layers": self.num_layers,
                "storage_format": self.storage_format,
                "clusters": [{"cluster_id": cid, "file": f, "experts": list(e)}
                             for cid, (f, e) in sorted(self.clusters.items())],
                "expert_to_cluster": {str(k): v for k, v in self.expert_to_cluster.items()}}

    def cluster_members(self, expert_id: int) -> List[int]:
        return list(self.clusters[self.expert_to_cluster[expert_id]][1])

    def cluster_file(self, cluster_id: int) -> str:
        return self.clusters[cluster_id][0]


def write_tensor_file(path: str, tensors: Dict[str, torch.Tensor]) -> None:
    """Write ``tensors`` (CPU) in the safetensors layout (keys sorted, data packed)."""
    header: Dict[str, Dict] = {}
    blobs = []
    off = 0
    for name in sorted(tensors):
        t = tensors[name].detach().cpu().contiguous()
        if t.dtype not in _ST_NAMES:
            raise TypeError(f"{name}: dtype {t.dtype} has no safetensors name")
        b = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _ST_NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)        # data section 8-byte aligned
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)
    os.replace(tmp, path)


def read_tensor_file(path: str, pin: bool = True) -> Dict[str, torch.Tensor]:
    """Read a safetensors-layout file with one sequential read into one (pinned)
    host buffer; returns zero-copy views of it."""
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(hlen))
        data_len = size - 8 - hlen
        buf = torch.empty(data_len, dtype=torch.uint8)
        if pin and torch.cuda.is_available():
            try:
                buf = buf.pin_memory()
            except RuntimeError:
                pass
        if data_len:
            view = memoryview(buf.numpy())
            got = 0
            while got < data_len:
                n = f.readinto(view[got:])
                if not n:
                    raise IOError(f"{path}: short read ({got} of {data_len} bytes)")
                got += n
    out: Dict[str, torch.Tensor] = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        dt = _ST_DTYPES[meta["dtype"]]
        lo, hi = meta["data_offsets"]
        shape = [int(s) for s in meta["shape"]]
        raw = buf[lo:hi]
        if hi <= lo:
            out[name] = torch.empty(shape, dtype=dt)
            continue
        try:
            out[name] = raw.view(dt).view(shape)
        except RuntimeError:  # offset not aligned to the element size: copy this one
            out[name] = raw.clone().view(dt).view(shape)
    return out


class ClusterStorage:
    """Reader/writer of cluster-packed expert weights (``chronos/io/storage.py:113-236``)."""

    def __init__(self, root_dir: str):
        self.root_dir = root_dir
        path = os.path.join(root_dir, MANIFEST_FILENAME)
        if not os.path.exists(path):
            raise FileNotFoundError(f"{MANIFEST_FILENAME} not found at {path}")
        with open(path) as f:
            self.manifest = ClusterManifest.from_dict(json.load(f))

    def load_cluster(self, cluster_id: int, dtype: Optional[torch.dtype] = None, pin: bool = True
                     ) -> Dict[int, Dict[int, Dict[str, torch.Tensor]]]:
        """``{expert: {layer: {param: tensor}}}`` of one cluster.  Without ``dtype``
        (or with the file's dtype) the tensors are views of one pinned buffer."""
        tensors = read_tensor_file(os.path.join(self.root_dir, self.manifest.cluster_file(cluster_id)), pin=pin)
        nested: Dict[int, Dict[int, Dict[str, torch.Tensor]]] = {}
        for key, t in tensors.items():
            parsed = _parse_key(key)
            if parsed is None:
                continue
            layer_id, expert_id, param = parsed
            if dtype is not None and t.dtype != dtype:
                t = t.to(dtype)
            nested.setdefault(expert_id, {}).setdefault(layer_id, {})[param] = t
        return nested

    def cluster_for_expert(self, expert_id: int) -> int:
        return self.manifest.expert_to_cluster[expert_id]

    def experts_in_cluster(self, cluster_id: int) -> List[int]:
        return list(self.manifest.clusters[cluster_id][1])

    @staticmethod
    def write_clusters(moe_layers, clusters: List[List[int]], output_dir: str, num_layers: int,
                       num_experts: int, dtype: torch.dtype = torch.float16) -> str:
        """One ``cluster_{id}.ctsr`` per cluster (every layer's copy of its experts)
        plus the manifest; returns the manifest path."""
        os.makedirs(output_dir, exist_ok=True)
        manifest_clusters: Dict[int, Tuple[str, List[int]]] = {}
        e2c: Dict[int, int] = {}
        for cid, cluster in enumerate(clusters):
            tensors: Dict[str, torch.Tensor] = {}
            for eid in cluster:
                e2c[int(eid)] = cid
                for li in range(min(num_layers, len(moe_layers))):
                    for pname, pval in moe_layers[li].experts[eid].state_dict().items():
                        tensors[_key(li, int(eid), pname)] = pval.detach().to(dtype=dtype).cpu().contiguous()
            fname = f"cluster_{cid}.ctsr"
            write_tensor_file(os.path.join(output_dir, fname), tensors)
            manifest_clusters[cid] = (fname, [int(e) for e in cluster])
        manifest = ClusterManifest(MANIFEST_VERSION, num_experts, num_layers, "safetensors",
                                   manifest_clusters, e2c)
        path = os.path.join(output_dir, MANIFEST_FILENAME)
        with open(path, "w") as f:
            json.dump(manifest.to_dict(), f, indent=2)
        return path

    @staticmethod
    def has_manifest(root_dir: str) -> bool:
        return os.path.exists(os.path.join(root_dir, MANIFEST_FILENAME))
