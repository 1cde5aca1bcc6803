"""Test helper: write a model as an MLX-layout safetensors checkpoint.

Tensor names, packing and dtypes follow what the reference loads
(src/serving/weights.rs:146-260, native/mlx_bridge.cpp:108-119): quantized
modules as `<name>.weight` (uint32 rows of LSB-first `bits`-bit values, expert
stacks shaped [experts, rows, words]), `<name>.scales` / `<name>.biases`
(bfloat16, one per group); vectors as float32. The values come from the FP64
oracle's synthetic model, so a checkpoint written here holds exactly the bytes
rs_qwen_weights_synthetic would generate for 4-bit g64 modules.
"""
from __future__ import annotations

import json
import struct

import numpy as np


def bf16_bits(values):
    """float32 values that are exactly bfloat16 -> their bf16 bits (checked)."""
    u = np.ascontiguousarray(values, np.float32).view(np.uint32)
    if np.any(u & 0xFFFF):
        raise ValueError("value is not a bfloat16")
    return (u >> 16).astype(np.uint16)


def to_bf16(values):
    """Round float32 to the nearest bfloat16 (ties to even), as float32."""
    u = np.ascontiguousarray(values, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def model_tensors(cfg, mtp=False):
    """(name, kind, rows, cols, mlx_shape) of every tensor of the model; kind is
    "q" (quantized matrix), "norm" (RMSNorm gain), "gnorm" (DeltaNet gated-norm
    gain), "conv", or "vec" (A_log, dt_bias)."""
    H, V = cfg.hidden, cfg.vocab
    kd, vd = cfg.key_heads * cfg.key_dim, cfg.value_heads * cfg.value_dim
    cd = 2 * kd + vd
    E, I, S, D = cfg.experts, cfg.intermediate, cfg.shared, cfg.head_dim
    out = [("language_model.model.embed_tokens", "q", V, H, None), ("language_model.lm_head", "q", V, H, None),
           ("language_model.model.norm.weight", "norm", H, 1, None)]

    def attention(p):
        return [(p + ".self_attn.q_proj", "q", cfg.q_heads * 2 * D, H, None),
                (p + ".self_attn.k_proj", "q", cfg.kv_heads * D, H, None),
                (p + ".self_attn.v_proj", "q", cfg.kv_heads * D, H, None),
                (p + ".self_attn.q_norm.weight", "norm", D, 1, None),
                (p + ".self_attn.k_norm.weight", "norm", D, 1, None),
                (p + ".self_attn.o_proj", "q", H, cfg.q_heads * D, None)]

    def moe(p):
        return [(p + ".mlp.gate", "q", E, H, None), (p + ".mlp.shared_expert_gate", "q", 1, H, None),
                (p + ".mlp.switch_mlp.gate_proj", "q", E * I, H, (E, I)),
                (p + ".mlp.switch_mlp.up_proj", "q", E * I, H, (E, I)),
                (p + ".mlp.switch_mlp.down_proj", "q", E * H, I, (E, H)),
                (p + ".mlp.shared_expert.gate_proj", "q", S, H, None),
                (p + ".mlp.shared_expert.up_proj", "q", S, H, None),
                (p + ".mlp.shared_expert.down_proj", "q", H, S, None)]

    for i in range(cfg.layers):
        p = f"language_model.model.layers.{i}"
        out += [(p + ".input_layernorm.weight", "norm", H, 1, None),
                (p + ".post_attention_layernorm.weight", "norm", H, 1, None)]
        if (i + 1) % cfg.interval == 0:
            out += attention(p)
        else:
            g = p + ".linear_attn"
            out += [(g + ".in_proj_qkv", "q", cd, H, None), (g + ".in_proj_z", "q", vd, H, None),
                    (g + ".in_proj_a", "q", cfg.value_heads, H, None),
                    (g + ".in_proj_b", "q", cfg.value_heads, H, None),
                    (g + ".conv1d.weight", "conv", cd, cfg.conv, None),
                    (g + ".A_log", "vec", cfg.value_heads, 1, None), (g + ".dt_bias", "vec", cfg.value_heads, 1, None),
                    (g + ".norm.weight", "gnorm", cfg.value_dim, 1, None), (g + ".out_proj", "q", H, vd, None)]
        out += moe(p)
    if mtp:
        m = "language_model.mtp"
        out += [(m + ".pre_fc_norm_embedding.weight", "norm", H, 1, None),
                (m + ".pre_fc_norm_hidden.weight", "norm", H, 1, None), (m + ".fc", "q", H, 2 * H, None),
                (m + ".layers.0.input_layernorm.weight", "norm", H, 1, None),
                (m + ".layers.0.post_attention_layernorm.weight", "norm", H, 1, None)]
        out += attention(m + ".layers.0") + moe(m + ".layers.0")
        out += [(m + ".norm.weight", "norm", H, 1, None)]
    return out


def quantize_rows(rng, rows, cols, bits, group):
    """Random affine data in another quantization: (packed LSB-first words,
    bf16-exact float32 scales, biases) whose values have std ~0.02."""
    q = rng.integers(0, 1 << bits, size=(rows, cols)).astype(np.uint64)
    levels = (1 << bits) - 1
    scales = to_bf16(np.full((rows, cols // group), 0.07 / levels, np.float32) *
                     rng.uniform(0.8, 1.2, size=(rows, cols // group)).astype(np.float32))
    biases = to_bf16(np.full((rows, cols // group), -0.035, np.float32))
    words = cols * bits // 32
    packed = np.zeros((rows, words), np.uint64)
    for c in range(cols):
        bit = c * bits
        w, sh = bit // 32, bit % 32
        packed[:, w] |= (q[:, c] << np.uint64(sh)) & np.uint64(0xFFFFFFFF)
        if sh + bits > 32:
            packed[:, w + 1] |= q[:, c] >> np.uint64(32 - sh)
    return packed.astype(np.uint32), scales, biases


def write_safetensors(path, tensors):
    """tensors: list of (name, numpy array, dtype string)."""
    header, blobs, off = {}, [], 0
    for name, arr, dt in tensors:
        raw = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    header["__metadata__"] = {"format": "mlx"}
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)


def checkpoint_tensors(cfg, model, overrides=None, shifted=False, mtp=False):
    """The model as (name, array, dtype) tensors. overrides: {module: (packed, scales, biases, bits)};
    shifted: store RMSNorm gains as offsets from 1 and conv1d weights in [channels, 1, taps] layout
    (the layout that marks such checkpoints)."""
    overrides = overrides or {}
    out = []
    for name, kind, rows, cols, shape3 in model_tensors(cfg, mtp):
        if kind == "q":
            if name in overrides:
                packed, sc, bi, _ = overrides[name]
            else:
                packed, sc, bi = model.qrows(name, 0, rows, cols)
            lead = shape3 if shape3 else (rows,)
            out.append((name + ".weight", packed.reshape(*lead, -1), "U32"))
            out.append((name + ".scales", bf16_bits(sc).reshape(*lead, -1), "BF16"))
            out.append((name + ".biases", bf16_bits(bi).reshape(*lead, -1), "BF16"))
        elif kind in ("norm", "gnorm"):
            gain = np.ones(rows, np.float32)
            if shifted and kind == "norm":
                gain = gain - 1.0
            out.append((name, gain, "F32"))
        elif kind == "conv":
            w = model.vector(name, rows * cols).reshape(rows, cols)
            out.append((name, w.reshape(rows, 1, cols) if shifted else w.reshape(rows, cols, 1), "F32"))
        else:
            out.append((name, model.vector(name, rows), "F32"))
    return out
