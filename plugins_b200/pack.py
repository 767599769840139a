"""A pack on disk: safetensors shards and config.json, read the way the plugin seam reads them.

The reference loads an EXL3 linear as the pack's ``<name>.trellis`` (int16 ``[in/16, out/16, n]``), ``<name>.suh``
(f16 ``[in]``) and ``<name>.svh`` (f16 ``[out]``) tensors through the host's ``Source`` (plugins/turboexl3_ds41/
plugin.zig:84-103), a bank as ``<prefix>.experts.<e>.<proj>`` for every expert its router ``<prefix>.gate.weight``
scores (plugin.zig:127-151), and claims the pack by the ``quantization_config`` block of config.json
(plugins/turboexl3_ds41/config.zig:13-61).  :class:`PackSource` is that ``Source`` over a directory of safetensors
files: it indexes every shard (``model.safetensors.index.json`` when present), memory-maps them and hands out
zero-copy numpy views, so ``quant.LoadContext(pack.block_json, pack.config_json, source=pack)`` uploads a real pack.

The safetensors format (a little-endian u64 header length, a JSON header of ``name -> {dtype, shape,
data_offsets}``, then the raw bytes) is read and written here directly; no third-party package is needed.
"""
from __future__ import annotations

import json
import mmap
import os
import struct

import numpy as np

# safetensors dtype names -> numpy (bf16 has no numpy type: its bits come back as uint16)
_TO_NP = {"F64": np.float64, "F32": np.float32, "F16": np.float16, "BF16": np.uint16, "I64": np.int64,
          "I32": np.int32, "I16": np.int16, "I8": np.int8, "U64": np.uint64, "U32": np.uint32, "U16": np.uint16,
          "U8": np.uint8, "BOOL": np.bool_}
_FROM_NP = {np.dtype(np.float64): "F64", np.dtype(np.float32): "F32", np.dtype(np.float16): "F16",
            np.dtype(np.int64): "I64", np.dtype(np.int32): "I32", np.dtype(np.int16): "I16", np.dtype(np.int8): "I8",
            np.dtype(np.uint64): "U64", np.dtype(np.uint32): "U32", np.dtype(np.uint16): "U16",
            np.dtype(np.uint8): "U8", np.dtype(np.bool_): "BOOL"}


class SafetensorsFile:
    """One safetensors file, memory-mapped; ``get(name)`` is a read-only zero-copy view."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        if len(self._mm) < 8:
            raise ValueError(f"{path}: not a safetensors file")
        (n,) = struct.unpack("<Q", self._mm[:8])
        if n > len(self._mm) - 8:
            raise ValueError(f"{path}: header length past the end of the file")
        header = json.loads(bytes(self._mm[8:8 + n]))
        self.metadata = header.pop("__metadata__", {}) or {}
        self._base = 8 + n
        self.entries = {}
        for name, e in header.items():
            dt = _TO_NP.get(e["dtype"])
            if dt is None:
                raise ValueError(f"{path}: {name} has the unsupported dtype {e['dtype']}")
            b0, b1 = e["data_offsets"]
            shape = tuple(int(s) for s in e["shape"])
            if b1 - b0 != int(np.prod(shape, dtype=np.int64)) * np.dtype(dt).itemsize or self._base + b1 > len(self._mm):
                raise ValueError(f"{path}: {name}'s byte range does not match its shape")
            self.entries[name] = (e["dtype"], dt, shape, b0, b1)

    def names(self):
        return self.entries.keys()

    def get(self, name: str) -> np.ndarray | None:
        e = self.entries.get(name)
        if e is None:
            return None
        _, dt, shape, b0, b1 = e
        return np.frombuffer(self._mm, dtype=dt, count=(b1 - b0) // np.dtype(dt).itemsize,
                             offset=self._base + b0).reshape(shape)

    def close(self):
        """Drops the file; arrays handed out keep the mapping alive until they are gone."""
        try:
            self._mm.close()
        except BufferError:
            pass  # views still exported: the mapping closes with the last of them
        finally:
            self._f.close()


def write_safetensors(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """Writes numpy arrays (C order, any _FROM_NP dtype) as one safetensors file; names sorted, data 8-byte aligned."""
    header, blobs, off = {}, [], 0
    for name in sorted(tensors):
        a = np.asarray(tensors[name])
        if not a.flags.c_contiguous:  # (ascontiguousarray would turn a 0-d array into 1-d)
            a = a.copy(order="C")
        dt = _FROM_NP.get(a.dtype)
        if dt is None:
            raise ValueError(f"{name}: dtype {a.dtype} has no safetensors name")
        raw = a.tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        pad = (-len(raw)) % 8
        blobs.append(raw + b"\0" * pad)
        off += len(raw) + pad
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((-len(h)) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


class PackSource:
    """A pack directory as the seam's ``Source``: ``pack(name)`` -> numpy array or None.

    ``block_json`` is config.json's ``quantization_config`` (the block the seam claims), ``config_json`` the whole
    config; ``stored_bytes`` the tensors' bytes (what ``bill`` sees as stored).
    """

    def __init__(self, directory: str):
        self.dir = directory
        cfg_path = os.path.join(directory, "config.json")
        self.config = json.load(open(cfg_path)) if os.path.exists(cfg_path) else {}
        qc = self.config.get("quantization_config") or (self.config.get("text_config") or {}).get("quantization_config")
        self.block = qc or {}
        self.files: dict[str, SafetensorsFile] = {}
        self.where: dict[str, str] = {}
        index = os.path.join(directory, "model.safetensors.index.json")
        if os.path.exists(index):
            weight_map = json.load(open(index)).get("weight_map", {})
            shards = sorted(set(weight_map.values()))
        else:
            weight_map = None
            shards = sorted(f for f in os.listdir(directory) if f.endswith(".safetensors"))
        for shard in shards:
            st = SafetensorsFile(os.path.join(directory, shard))
            self.files[shard] = st
            for name in st.names():
                if weight_map is not None and weight_map.get(name) != shard:
                    continue
                if name in self.where:
                    raise ValueError(f"{name} is in both {self.where[name]} and {shard}")
                self.where[name] = shard

    @property
    def block_json(self) -> str:
        return json.dumps(self.block)

    @property
    def config_json(self) -> str:
        return json.dumps(self.config)

    @property
    def stored_bytes(self) -> int:
        return sum(e[4] - e[3] for f in self.files.values() for e in f.entries.values())

    def names(self):
        return self.where.keys()

    def __call__(self, name: str) -> np.ndarray | None:
        shard = self.where.get(name)
        return None if shard is None else self.files[shard].get(name)

    def close(self):
        for f in self.files.values():
            f.close()
        self.files.clear()
        self.where.clear()


def write_pack(directory: str, tensors: dict, config: dict, shards: int = 1) -> None:
    """A pack for tests and tools: tensors spread over `shards` safetensors files (with an index when more than one)
    and config.json."""
    os.makedirs(directory, exist_ok=True)
    names = sorted(tensors)
    per = (len(names) + shards - 1) // max(shards, 1)
    weight_map = {}
    for i in range(shards):
        part = names[i * per:(i + 1) * per]
        fname = "model.safetensors" if shards == 1 else f"model-{i + 1:05d}-of-{shards:05d}.safetensors"
        write_safetensors(os.path.join(directory, fname), {n: tensors[n] for n in part})
        weight_map.update({n: fname for n in part})
    if shards > 1:
        json.dump({"metadata": {}, "weight_map": weight_map},
                  open(os.path.join(directory, "model.safetensors.index.json"), "w"))
    json.dump(config, open(os.path.join(directory, "config.json"), "w"))
