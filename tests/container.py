"""Write a weight container in the layout the reference's loader reads (test
helper): safetensors shards (8-byte little-endian header length, a JSON
header of name -> dtype / shape / data_offsets, then the data),
model.safetensors.index.json with the weight_map, and a flat config.json.
Container names are the checkpoint names minus "model.language_model."
(c/st.h:25-80, c/gmodel.h:373-480; the converter's output layout is
described in the reference's tests/m1/README.md)."""
import json
import os
import struct

import numpy as np

ST_DTYPE = {"bf16": "BF16", "f32": "F32", "scale": "F32", "e4m3": "F8_E4M3"}


def write_shard(path, tensors):
    """tensors: list of (name, safetensors dtype, shape, numpy array)."""
    header, blobs, off = {}, [], 0
    for name, dt, shape, arr in tensors:
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)             # the header is padded to 8 bytes, as safetensors writers do
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_container(root, kw, W, specs, n_shards=2):
    """Container of the weights W (name -> array) described by specs
    (tensor_specs(kw) rows: name, shape, numpy dtype, kind) under root/, the
    tensors spread round-robin over n_shards shards; config.json is the flat
    layout with explicit layer lists."""
    os.makedirs(root, exist_ok=True)
    groups = [[] for _ in range(n_shards)]
    for i, (name, shape, _, kind) in enumerate(specs):
        groups[i % n_shards].append((name, ST_DTYPE[kind], shape, W[name]))
    weight_map, total = {}, 0
    for i, g in enumerate(groups):
        fname = f"apus-{i + 1:05d}.safetensors"
        write_shard(os.path.join(root, fname), g)
        for name, _, _, arr in g:
            weight_map[name] = fname
            total += np.asarray(arr).nbytes
    with open(os.path.join(root, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f)
    cfg = dict(kw)
    L = kw["num_hidden_layers"]
    cfg["layer_types"] = ["deepseek_sparse_attention" if kw["layer_is_dsa"][i] else "linear_attention"
                          for i in range(L)]
    cfg["mlp_layer_types"] = ["sparse" if kw["mlp_is_sparse"][i] else "dense" for i in range(L)]
    cfg.pop("layer_is_dsa", None)
    cfg.pop("mlp_is_sparse", None)
    with open(os.path.join(root, "config.json"), "w") as f:
        json.dump(cfg, f)
    return os.path.join(root, "config.json")
