"""Checkpoint ingestion on the host (no GPU): MLX-layout safetensors shards
are read by rs_mlx_weights_load and every tensor comes back byte for byte from
rs_mlx_weight_bytes, with the reference's dtype and shape checks
(native/mlx_bridge.cpp:108-119, 177-187; src/serving/weights.rs:146-260)."""
import ctypes as C
import struct

import numpy as np
import pytest

from checkpoint_util import checkpoint_tensors, quantize_rows, write_safetensors

DTYPE = {"F32": 0, "I32": 1, "U32": 2, "F16": 3, "BF16": 4}


def test_shards_round_trip_bit_for_bit(pkg, O, tmp_path):
    cfg = O.config0()
    model = O.Model(cfg, 13)
    rng = np.random.default_rng(2)
    ov = {"language_model.model.layers.1.mlp.gate": quantize_rows(rng, cfg.experts, cfg.hidden, 8, 64) + (8,)}
    tensors = checkpoint_tensors(cfg, model, overrides=ov, shifted=True)
    half = len(tensors) // 2
    write_safetensors(tmp_path / "a.safetensors", tensors[:half])
    write_safetensors(tmp_path / "b.safetensors", tensors[half:])
    store = pkg.WeightStore()
    store.load(tmp_path / "a.safetensors").load(tmp_path / "b.safetensors")
    store.quant("language_model.model.layers.1.mlp.gate", 64, 8)
    lib = pkg.load()
    for name, arr, dt in tensors:
        raw = np.ascontiguousarray(arr).tobytes()
        for off, cnt in ((0, len(raw)), (len(raw) // 3, len(raw) - len(raw) // 3)):
            got = store.weight_bytes(name, off, cnt, DTYPE[dt])
            assert got == raw[off:off + cnt], name
        shape = (C.c_int32 * len(arr.shape))(*arr.shape)
        buf = (C.c_uint8 * 4)()
        err = C.create_string_buffer(256)
        wrong = DTYPE["F16"] if dt != "F16" else DTYPE["F32"]
        assert lib.rs_mlx_weight_bytes(store.h, name.encode(), shape, len(arr.shape), wrong, 0, buf, 4, err, 256) == -1
        assert b"bounds/type" in err.value
    store.close()


def test_loader_rejects_malformed_shards(pkg, tmp_path):
    good = [("a.weight", np.arange(8, dtype=np.uint32).reshape(2, 4), "U32")]
    write_safetensors(tmp_path / "one.safetensors", good)
    store = pkg.WeightStore().load(tmp_path / "one.safetensors")
    with pytest.raises(pkg.NativeError, match="duplicate native parameter"):
        store.load(tmp_path / "one.safetensors")
    store.close()
    bad = tmp_path / "bad.safetensors"
    header = b'{"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 32]}}'
    bad.write_bytes(struct.pack("<Q", len(header)) + header + b"\0" * 16)  # offsets past the data
    with pytest.raises(pkg.NativeError, match="offsets outside shard"):
        pkg.WeightStore().load(bad)
    header = b'{"x": {"dtype": "F64", "shape": [1], "data_offsets": [0, 8]}}'
    bad.write_bytes(struct.pack("<Q", len(header)) + header + b"\0" * 8)
    with pytest.raises(pkg.NativeError, match="unsupported parameter dtype"):
        pkg.WeightStore().load(bad)
    header = (b'{"x": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},'
              b' "y": {"dtype": "F32", "shape": [2], "data_offsets": [4, 12]}}')
    bad.write_bytes(struct.pack("<Q", len(header)) + header + b"\0" * 12)
    with pytest.raises(pkg.NativeError, match="overlapping"):
        pkg.WeightStore().load(bad)
    bad.write_bytes(struct.pack("<Q", 9) + b'{"x": [1,')
    with pytest.raises(pkg.NativeError, match="safetensors header"):
        pkg.WeightStore().load(bad)
    with pytest.raises(pkg.NativeError):
        pkg.WeightStore().quant("m", 48, 4)  # the reference's quantization bounds
