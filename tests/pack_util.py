"""A small seeded Hugging Face-style snapshot for the blob-packer tests.

Same tensor names and layer pattern as Qwen3.5 ([3 x linear_attention, 1 x
full_attention]), tiny dimensions.  It exercises what the packer must get
right: BF16 widening, F16 and F32 inputs, the "model.language_model." prefix,
vision and MTP tensors to skip, two shard files, an all-zero matrix row
(scale 1.0) and a row of exact rounding ties (rint half to even).
"""

from __future__ import annotations

import json
import os
import struct

import numpy as np

from qwen_fpga_b200 import synth

TINY = {
    "hidden_size": 64, "num_hidden_layers": 4,
    "layer_types": ["linear_attention"] * 3 + ["full_attention"],
    "head_dim": 32, "num_attention_heads": 2, "num_key_value_heads": 1,
    "intermediate_size": 96, "vocab_size": 300, "rms_norm_eps": 1e-06,
    "linear_num_value_heads": 2, "linear_num_key_heads": 2,
    "linear_key_head_dim": 16, "linear_value_head_dim": 16, "linear_conv_kernel_dim": 4,
    "rope_parameters": {"rope_theta": 10000000, "partial_rotary_factor": 0.25, "rope_type": "default"},
}


def _bf16(a: np.ndarray) -> bytes:
    """float32 -> bfloat16 bytes (round to nearest even on the dropped half)."""
    u = a.astype(np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16).tobytes()


def _write_safetensors(path: str, tensors: list[tuple[str, str, tuple, bytes]]):
    hdr, blobs, off = {"__metadata__": {"format": "pt"}}, [], 0
    for name, dtype, shape, raw in tensors:
        hdr[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(hdr).encode()
    h += b" " * ((-len(h)) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def make_tiny_snapshot(d: str, seed: int = 3) -> str:
    """Write config.json and two *.safetensors files into d; returns d."""
    os.makedirs(d, exist_ok=True)
    cfg = dict(TINY)
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump({"model_type": "qwen3_5", "text_config": cfg}, f, indent=2)
    shapes = synth.tensor_shapes(cfg)
    rng = np.random.default_rng(seed)
    items = []
    for i, name in enumerate(synth.tensor_order(cfg)):
        w = (rng.standard_normal(shapes[name]) * 0.02).astype(np.float32)
        if name == "layers.0.linear_attn.in_proj_z.weight":
            w[3] = 0.0                                    # all-zero row: scale 1.0, q = 0
        if name == "layers.1.mlp.down_proj.weight":
            w[5] = 0.0
            w[5, :6] = [127.0, 0.5, 1.5, 2.5, -0.5, -3.5]  # scale 1.0: exact ties for rint
        if name.endswith(("A_log", "dt_bias")):
            items.append((name, "F32", w.shape, w.tobytes()))
        elif name.endswith("conv1d.weight"):
            items.append((name, "F16", w.shape, w.astype(np.float16).tobytes()))
        else:
            items.append((name, "BF16", w.shape, _bf16(w)))
    items = [("model.language_model." + n, dt, sh, raw) for n, dt, sh, raw in items]
    extra = [("model.visual.blocks.0.attn.qkv.weight", "BF16", (4, 4), _bf16(np.ones((4, 4), np.float32))),
             ("mtp.fc.weight", "F32", (2, 2), np.ones((2, 2), np.float32).tobytes())]
    half = len(items) // 2
    _write_safetensors(os.path.join(d, "model-00001-of-00002.safetensors"), items[:half] + extra[:1])
    _write_safetensors(os.path.join(d, "model-00002-of-00002.safetensors"), items[half:] + extra[1:])
    return d
