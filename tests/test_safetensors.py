"""Safetensors checkpoint ingest, host side (no GPU): the header index of
msgl_safetensors_index over a directory of shards, and its errors on malformed files.

`write_safetensors` writes the published safetensors layout (8-byte little-endian header size,
JSON header name -> {dtype, shape, data_offsets}, then the raw data); the GPU test of
msgl_model_load_safetensors (test_weights_gpu.py) uses it too.
"""
import ctypes as C
import json
import os
import struct

import numpy as np

import msgl

ERR_INVALID_ARG = 1


def _bytes(a, dtype):
    a = np.ascontiguousarray(a, dtype=np.float32)
    if dtype == "F32":
        return a.tobytes()
    if dtype == "F16":
        return a.astype(np.float16).tobytes()
    # BF16: the values are bf16-representable, so the high half of the fp32 bits is exact
    return (a.view(np.uint32) >> 16).astype(np.uint16).tobytes()


def write_safetensors(path, tensors, metadata=None):
    """tensors: {name: (float32 array, dtype in BF16 / F16 / F32)}."""
    header, blobs, off = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, (a, dt) in tensors.items():
        b = _bytes(a, dt)
        header[name] = {"dtype": dt, "shape": list(np.shape(a)), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def index(d):
    n, b = C.c_int64(0), C.c_int64(0)
    rc = msgl.lib().msgl_safetensors_index(os.fsencode(str(d)), C.addressof(n), C.addressof(b))
    return rc, n.value, b.value


def test_index_counts_every_shard(tmp_path):
    rng = np.random.default_rng(0)
    a, b, c = (rng.standard_normal(s).astype(np.float32) for s in ((3, 4), (7,), (2, 2, 2)))
    write_safetensors(tmp_path / "model-00001-of-00002.safetensors",
                      {"x.weight": (a, "BF16"), "y.weight": (b, "F32")}, {"format": "pt"})
    write_safetensors(tmp_path / "model-00002-of-00002.safetensors", {"z.weight": (c, "F16")})
    (tmp_path / "config.json").write_text("{}")  # other files are ignored
    rc, n, nbytes = index(tmp_path)
    assert rc == 0 and n == 3 and nbytes == 12 * 2 + 7 * 4 + 8 * 2


def test_index_rejects_malformed_files(tmp_path):
    L = msgl.lib()
    assert index(tmp_path / "missing")[0] == ERR_INVALID_ARG
    assert index(tmp_path)[0] == ERR_INVALID_ARG  # no shard
    assert b"no .safetensors" in L.msgl_last_error()
    bad = tmp_path / "bad.safetensors"
    h = b'{"w": {"dtype": "BF16", "shape": [4], "data_offsets": [0, 8]'  # unterminated
    bad.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 8)
    assert index(tmp_path)[0] == ERR_INVALID_ARG
    assert b"safetensors header" in L.msgl_last_error()
    h = json.dumps({"w": {"dtype": "BF16", "shape": [4], "data_offsets": [0, 6]}}).encode()
    bad.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 8)  # 4 bf16 values are 8 bytes
    assert index(tmp_path)[0] == ERR_INVALID_ARG
    assert b"does not match its shape" in L.msgl_last_error()
    h = json.dumps({"w": {"dtype": "BF16", "shape": [4], "data_offsets": [0, 8]}}).encode()
    bad.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 4)  # data cut short
    assert index(tmp_path)[0] == ERR_INVALID_ARG
    assert b"past the end" in L.msgl_last_error()
    bad.write_bytes(struct.pack("<Q", 1 << 40) + b"{}")  # header size beyond the file
    assert index(tmp_path)[0] == ERR_INVALID_ARG
    h = '{"w\\u00e9\\n": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 4]}}'.encode()
    bad.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 4)  # escapes in names are fine
    assert index(tmp_path)[:2] == (0, 1)
