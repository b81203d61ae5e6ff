"""safetensors files and MLX-affine checkpoint directories.

The reference loads its checkpoints through ``mlx_lm.utils.load_model``
(``spark_mlx_llm/loader.py:65-120``): ``config.json`` plus ``model*.safetensors``
shards whose quantized linears are MLX affine triples ``<name>.weight`` (uint32
words, element j of a word at bits [j*b, j*b+b)), ``<name>.scales`` and
``<name>.biases`` (one per group of ``group_size`` along K). This module reads
(and, for tests and converters, writes) that format with NumPy alone - the
safetensors layout is an 8-byte little-endian header length, a JSON header
``{name: {dtype, shape, data_offsets}}`` and the raw little-endian tensor bytes.
"""

import glob
import json
import os
import struct

import numpy as np
import torch

__all__ = ["read_safetensors", "write_safetensors", "load_checkpoint_dir", "to_torch"]

# safetensors dtype -> (numpy storage dtype, torch dtype); BF16 is stored as its 16 bits
_DTYPES = {
    "BF16": (np.uint16, torch.bfloat16),
    "F16": (np.float16, torch.float16),
    "F32": (np.float32, torch.float32),
    "U32": (np.uint32, torch.int32),   # packed codes: the same 32 bits as int32
    "I32": (np.int32, torch.int32),
    "I8": (np.int8, torch.int8),
    "U8": (np.uint8, torch.uint8),
    "I64": (np.int64, torch.int64),
    "BOOL": (np.bool_, torch.bool),
}


def read_safetensors(path):
    """``{name: (dtype_name, numpy array)}`` of one safetensors file (arrays are
    read-only views of a memory map; BF16 arrives as uint16 bits)."""
    with open(path, "rb") as f:
        head = f.read(8)
        if len(head) != 8:
            raise ValueError(f"{path}: not a safetensors file")
        (n,) = struct.unpack("<Q", head)
        if n <= 0 or n > 100 << 20:
            raise ValueError(f"{path}: bad safetensors header length {n}")
        header = json.loads(f.read(n))
    data = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + n)
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        dt = meta["dtype"]
        if dt not in _DTYPES:
            raise ValueError(f"{path}: tensor {name!r} has unsupported dtype {dt}")
        np_dt = _DTYPES[dt][0]
        b0, b1 = meta["data_offsets"]
        shape = tuple(int(s) for s in meta["shape"])
        count = int(np.prod(shape)) if shape else 1
        if b1 - b0 != count * np.dtype(np_dt).itemsize or b1 > data.size:
            raise ValueError(f"{path}: tensor {name!r} has inconsistent offsets")
        out[name] = (dt, np.frombuffer(data, dtype=np_dt, count=count, offset=b0).reshape(shape))
    return out


def write_safetensors(path, tensors, metadata=None):
    """Write ``{name: (dtype_name, numpy array)}`` (BF16 given as uint16 bits) in
    the safetensors layout, tensors in name order."""
    header, blobs, offset = {}, [], 0
    for name in sorted(tensors):
        dt, arr = tensors[name]
        np_dt = _DTYPES[dt][0]
        arr = np.ascontiguousarray(np.asarray(arr).astype(np_dt, copy=False))
        raw = arr.tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [offset, offset + len(raw)]}
        blobs.append(raw)
        offset += len(raw)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    text = json.dumps(header, separators=(",", ":")).encode()
    text += b" " * (-len(text) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for raw in blobs:
            f.write(raw)


def load_checkpoint_dir(path):
    """``(config dict, {name: (dtype, array)})`` of a checkpoint directory:
    ``config.json`` and every ``model*.safetensors`` shard
    (``loader.py:14-24`` allow-patterns; the reference resolves a hub id, this
    takes a local directory)."""
    path = os.fspath(path)
    if not os.path.isdir(path):
        raise NotADirectoryError(f"Model path must be a directory: {path}")
    cfg_path = os.path.join(path, "config.json")
    if not os.path.exists(cfg_path):
        raise FileNotFoundError(f"{cfg_path} does not exist")
    with open(cfg_path) as f:
        config = json.load(f)
    shards = sorted(glob.glob(os.path.join(path, "model*.safetensors")))
    if not shards:
        raise FileNotFoundError(f"no model*.safetensors in {path}")
    weights = {}
    for shard in shards:
        for name, value in read_safetensors(shard).items():
            if name in weights:
                raise ValueError(f"tensor {name!r} appears in more than one shard")
            weights[name] = value
    return config, weights


def to_torch(entry, device):
    """A ``(dtype, array)`` entry as a torch tensor on ``device`` (bit-exact)."""
    dt, arr = entry
    arr = np.ascontiguousarray(arr)
    if dt == "BF16":
        return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16).to(device)
    if dt == "U32":
        return torch.from_numpy(arr.view(np.int32).copy()).to(device)
    return torch.from_numpy(arr.copy()).to(device)
