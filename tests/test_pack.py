"""The C++ blob packer (qwen_pack_blob, host only) against the reference packer.

tests/golden/pack_tiny.json holds the unmodified reference packer's output
(scripts/pack_weights.py with golden/loader.py and golden/quant.py, run by
tests/golden/make_pack_golden.py) on the seeded snapshot of tests/pack_util.py.
Bar: the same blob byte for byte, the same manifest, and the flat index
emit_weight_index.py would write from it.
"""

import hashlib
import json
import os

import pytest

from pack_util import make_tiny_snapshot

HERE = os.path.dirname(os.path.abspath(__file__))


def _pack(snap, out):
    from qwen_fpga_b200 import api
    api.pack_blob(snap, out)


@pytest.fixture(scope="module")
def packed(tmp_path_factory):
    d = tmp_path_factory.mktemp("pack")
    snap = make_tiny_snapshot(str(d / "snap"))
    out = str(d / "tiny_int8.bin")
    _pack(snap, out)
    return out


def test_blob_matches_reference_packer(packed):
    fx = json.load(open(os.path.join(HERE, "golden", "pack_tiny.json")))
    blob = open(packed, "rb").read()
    assert len(blob) == fx["blob_bytes"]
    assert hashlib.sha256(blob).hexdigest() == fx["blob_sha256"]


def test_manifest_and_index_match(packed):
    from qwen_fpga_b200 import synth
    fx = json.load(open(os.path.join(HERE, "golden", "pack_tiny.json")))["manifest"]
    stem = os.path.splitext(packed)[0]
    man = json.load(open(stem + ".manifest.json"))
    assert man == fx
    # the flat index is the manifest's lines (scripts/emit_weight_index.py:16-24)
    lines = open(stem + ".idx").read().splitlines()
    assert lines == synth.index_lines(man)


def test_missing_or_extra_tensors_are_rejected(tmp_path):
    from qwen_fpga_b200 import api
    snap = make_tiny_snapshot(str(tmp_path / "snap"))
    os.remove(os.path.join(snap, "model-00002-of-00002.safetensors"))
    with pytest.raises(api.QwenError) as e:
        _pack(snap, str(tmp_path / "x.bin"))
    assert e.value.code == 2 and "missing" in str(e.value)
    with pytest.raises(api.QwenError):
        _pack(str(tmp_path / "nowhere"), str(tmp_path / "y.bin"))
