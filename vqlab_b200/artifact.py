"""Load a VQLab artifact's VQ layers straight into B200 modules.

An artifact is a directory (src/vqlab/selftest/synthetic_model.py:44-130,
src/vqlab/bundle/add_model_file.py, src/vqlab/runtime/vq_switch.py:4989-5013):

  config.json                     `vq_modules` (switch layers: prefix -> {experts,
                                  out, in, group, dim, k, pack_bits?}) and/or
                                  `vq_linear` (dense layers: prefix -> {out, in,
                                  group, dim, k, pack_bits?})
  model.safetensors.index.json    `weight_map`: tensor key -> shard file
  *.safetensors                   {p}.codes, {p}.codebook, {p}.vq_scales; a
                                  SKIPZERO layer carries {p}.sz_codes,
                                  {p}.sz_scales, {p}.sz_rowmask instead

`load_vq_layers` returns {prefix: VQSwitchLinear | VQLinear}; SKIPZERO layers
get their row table from the live-row mask (skipzero_row_table).  The
safetensors reader and writer here follow the published file format (8-byte
little-endian header length, JSON header of dtype / shape / data_offsets,
then the raw little-endian tensor bytes); the `safetensors` package is not
needed.
"""
from __future__ import annotations

import json
import pathlib
import struct
from typing import Dict, Iterable, Optional

import numpy as np
import torch

from .vq_dense import VQLinear
from .vq_switch import VQSwitchLinear, skipzero_row_table

# safetensors dtype names <-> torch dtypes (the ones VQ artifacts use)
_ST_TO_TORCH = {"U8": torch.uint8, "I8": torch.int8, "I16": torch.int16, "U16": torch.uint16,
                "I32": torch.int32, "U32": torch.uint32, "I64": torch.int64, "F16": torch.float16,
                "BF16": torch.bfloat16, "F32": torch.float32, "F64": torch.float64, "BOOL": torch.bool}
_TORCH_TO_ST = {v: k for k, v in _ST_TO_TORCH.items()}
_ST_ITEMSIZE = {"U8": 1, "I8": 1, "BOOL": 1, "I16": 2, "U16": 2, "F16": 2, "BF16": 2, "I32": 4, "U32": 4, "F32": 4,
                "I64": 8, "F64": 8}


def read_safetensors_header(path) -> dict:
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        if n > (1 << 28):
            raise ValueError(f"{path}: implausible safetensors header length {n}")
        return json.loads(f.read(n))


def read_safetensors(path, keys: Optional[Iterable[str]] = None) -> Dict[str, torch.Tensor]:
    """Tensors of one safetensors file as CPU torch tensors (all keys, or `keys`)."""
    path = str(path)
    hdr = read_safetensors_header(path)
    base = 8 + struct.unpack("<Q", open(path, "rb").read(8))[0]
    want = set(keys) if keys is not None else None
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for k, meta in hdr.items():
        if k == "__metadata__" or (want is not None and k not in want):
            continue
        dt = meta["dtype"]
        if dt not in _ST_TO_TORCH:
            raise ValueError(f"{path}: tensor {k} has unsupported dtype {dt}")
        a, b = meta["data_offsets"]
        shape = [int(s) for s in meta["shape"]]
        if b - a != int(np.prod(shape, dtype=np.int64)) * _ST_ITEMSIZE[dt]:
            raise ValueError(f"{path}: tensor {k}: byte range does not match its shape")
        if b == a:
            out[k] = torch.empty(shape, dtype=_ST_TO_TORCH[dt])
            continue
        raw = torch.from_numpy(np.array(mm[base + a:base + b]))  # copy out of the map
        out[k] = raw.view(_ST_TO_TORCH[dt]).reshape(shape)
    if want is not None and want - out.keys():
        raise KeyError(f"{path}: missing tensors {sorted(want - out.keys())}")
    return out


def write_safetensors(path, tensors: Dict[str, torch.Tensor], metadata: Optional[dict] = None) -> None:
    """Write CPU tensors in the safetensors layout (keys sorted, 8-byte aligned data)."""
    hdr, blobs, off = {}, [], 0
    for k in sorted(tensors):
        t = tensors[k].detach().cpu().contiguous()
        if t.dtype not in _TORCH_TO_ST:
            raise ValueError(f"unsupported dtype {t.dtype} for {k}")
        b = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        hdr[k] = {"dtype": _TORCH_TO_ST[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        hdr["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(hdr, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


class Artifact:
    """A VQLab artifact directory: config and tensor index."""

    def __init__(self, root):
        self.root = pathlib.Path(root)
        self.config = json.loads((self.root / "config.json").read_text())
        idx = self.root / "model.safetensors.index.json"
        if idx.exists():
            self.index = json.loads(idx.read_text())["weight_map"]
        else:
            self.index = {}
            for f in sorted(self.root.glob("*.safetensors")):
                for k in read_safetensors_header(f):
                    if k != "__metadata__":
                        self.index[k] = f.name

    def modules(self) -> Dict[str, tuple]:
        """prefix -> ("switch" | "dense", meta) for every VQ layer the config declares."""
        out = {p: ("switch", m) for p, m in (self.config.get("vq_modules") or {}).items()}
        out.update({p: ("dense", m) for p, m in (self.config.get("vq_linear") or {}).items()})
        return out

    def tensors(self, keys: Iterable[str]) -> Dict[str, torch.Tensor]:
        by_file: Dict[str, list] = {}
        for k in keys:
            if k not in self.index:
                raise KeyError(f"{self.root}: no tensor {k} in the artifact index")
            by_file.setdefault(self.index[k], []).append(k)
        out = {}
        for f, ks in by_file.items():
            out.update(read_safetensors(self.root / f, ks))
        return out


def _pack_bits(meta: dict, codes: torch.Tensor, k: int) -> int:
    """BITS of a layer: the config's pack_bits, else packed uint32 words imply bit_length(K-1) (vq_switch.py:5236-5248)."""
    if meta.get("pack_bits"):
        return int(meta["pack_bits"])
    if codes.dtype in (torch.int32, torch.uint32):
        return int(k - 1).bit_length()
    return 0


def load_vq_layers(root, device="cuda", only: Optional[Iterable[str]] = None) -> Dict[str, torch.nn.Module]:
    """{prefix: VQSwitchLinear | VQLinear} for the artifact's VQ layers (or the `only` prefixes)."""
    art = Artifact(root)
    mods = art.modules()
    if only is not None:
        mods = {p: mods[p] for p in only}
    out = {}
    for p, (kind, meta) in mods.items():
        sz = (p + ".sz_rowmask") in art.index
        keys = [p + ".codebook"] + ([p + ".sz_codes", p + ".sz_scales", p + ".sz_rowmask"] if sz
                                    else [p + ".codes", p + ".vq_scales"])
        t = art.tensors(keys)
        cb = t[p + ".codebook"]
        codes = t[p + ".sz_codes"] if sz else t[p + ".codes"]
        sc = t[p + ".sz_scales"] if sz else t[p + ".vq_scales"]
        if codes.dtype == torch.uint32:
            codes = codes.view(torch.int32)  # the kernels read the words' bits
        if codes.dtype == torch.uint16:
            codes = codes.view(torch.int16)
        bits = _pack_bits(meta, codes, int(cb.shape[0]))
        G = int(meta.get("group", meta.get("group_size", 64)))
        IN = int(meta["in"])
        dev = torch.device(device)
        codes, cb, sc = codes.to(dev), cb.to(dev), sc.to(dev)
        if kind == "switch":
            rt = None
            if sz:
                rt = skipzero_row_table(t[p + ".sz_rowmask"], int(meta["experts"]), int(meta["out"])).to(dev)
            out[p] = VQSwitchLinear(codes, cb, sc, group_size=G, pack_bits=bits, in_features=IN if bits else None,
                                    row_table=rt)
        else:
            if sz:
                raise NotImplementedError(f"{p}: SKIPZERO is a switch-layer format")
            out[p] = VQLinear(codes, cb, sc, group_size=G, pack_bits=bits, in_features=IN if bits else None)
    return out
