"""Writer for the safetensors format (8-byte little-endian header length, JSON header of
name -> dtype / shape / data_offsets, raw little-endian data), used by the tests to put
oracle weights on disk the way a Hugging Face checkpoint stores them."""
import json
import os
import struct

import numpy as np

_DT = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.float64): "F64"}


def write_safetensors(path, tensors, bf16=False):
    """``tensors``: name -> float array; with ``bf16`` the arrays are stored as BF16
    (round to nearest even of the f32 value)."""
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        if bf16:
            u = a.astype(np.float32).view(np.uint32).astype(np.uint64)
            b = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
            raw, dt = b.tobytes(), "BF16"
        else:
            raw, dt = a.tobytes(), _DT[a.dtype]
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    header["__metadata__"] = {"format": "pt"}
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for raw in blobs:
            f.write(raw)


def write_sharded(model_dir, tensors, nshards=2, bf16=False):
    """Shards model-0000k-of-0000n.safetensors plus model.safetensors.index.json."""
    names = list(tensors)
    parts = [names[i::nshards] for i in range(nshards)]
    wmap = {}
    for k, part in enumerate(parts):
        fn = f"model-{k + 1:05d}-of-{nshards:05d}.safetensors"
        write_safetensors(os.path.join(model_dir, fn), {n: tensors[n] for n in part}, bf16)
        wmap.update({n: fn for n in part})
    with open(os.path.join(model_dir, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": 0}, "weight_map": wmap}, f)
