"""The C++ blob packer on a full-size snapshot, closing the loop with the
decoder.

A float32 Hugging Face-style snapshot of the seed-1234 random-init
Qwen3.5-0.8B (the same draws, in the same order, as the blob every other test
decodes: qwen_fpga_b200.synth.write_blob) is packed with qwen_pack_blob
(scripts/pack_weights.py's layout, golden/quant.py's quantiser).  Bar: the
packed blob is byte-identical to the seeded blob the golden fixtures were
generated from (config0.npz blob_sha256), and the decoder, loading the blob
and index the packer wrote, reproduces the golden's first greedy argmaxes.

GPU-marked: it needs the device for the decode and writes ~3 GB of snapshot,
more than the CPU suite's budget allows.
"""

import hashlib
import json
import os
import struct

import numpy as np
import pytest

from golden_util import fixture

pytestmark = pytest.mark.gpu


def write_f32_snapshot(d, seed=1234, std=0.02):
    """config.json + one model.safetensors of F32 tensors, the draws of synth.write_blob."""
    from qwen_fpga_b200 import synth
    os.makedirs(d, exist_ok=True)
    cfg = synth.model_config()
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump({"model_type": "qwen3_5", "text_config": cfg}, f)
    shapes = synth.tensor_shapes(cfg)
    order = [t["name"] for t in synth.layout(cfg)["tensors"]]
    hdr, off = {"__metadata__": {"format": "pt"}}, 0
    for n in order:
        nb = 4 * int(np.prod(shapes[n]))
        hdr["model.language_model." + n] = {"dtype": "F32", "shape": list(shapes[n]),
                                            "data_offsets": [off, off + nb]}
        off += nb
    h = json.dumps(hdr).encode()
    h += b" " * ((-len(h)) % 8)
    rng = np.random.default_rng(seed)
    with open(os.path.join(d, "model.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for n in order:
            f.write((rng.standard_normal(shapes[n], np.float32) * std).astype("<f4").tobytes())
    return d


def test_full_snapshot_packs_to_the_seeded_blob_and_decodes(tmp_path):
    from qwen_fpga_b200 import api
    fx = fixture("config0.npz")
    snap = write_f32_snapshot(str(tmp_path / "snap"))
    out = str(tmp_path / "qwen35_int8.bin")
    idx = api.pack_blob(snap, out)
    os.remove(os.path.join(snap, "model.safetensors"))
    h = hashlib.sha256()
    with open(out, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    assert h.hexdigest() == str(fx["blob_sha256"])
    with api.Decoder(out, idx, max_ctx=16) as d:
        for i, t in enumerate(fx["prompt"].tolist()[:3]):
            am, _ = d.decode_step(t, want_logits=False)
            assert am == int(fx["argmax"][i]), i
