"""Fixture for the C++ blob packer: the UNMODIFIED reference packer's output on
the small seeded snapshot of tests/pack_util.py.

Runs in the build container only: it imports scripts/pack_weights.py (and
through it golden/loader.py and golden/quant.py) from the reference checkout,
points its snapshot lookup at the generated snapshot and runs its main().
The test (tests/test_pack.py) compares libqwenb200's qwen_pack_blob with the
digests stored here.

    python tests/golden/make_pack_golden.py --ref PATH   (or QWEN_REF=PATH)

Writes tests/golden/pack_tiny.json: the blob's sha256 and size, and the
manifest's config and tensor entries.
"""

from __future__ import annotations

import argparse
import hashlib
import io
import json
import os
import sys
import tempfile
from contextlib import redirect_stdout

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))                  # tests/ (pack_util)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))  # the repository (qwen_fpga_b200)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("QWEN_REF"),
                    help="the reference checkout (or set QWEN_REF)")
    args = ap.parse_args()
    from pack_util import make_tiny_snapshot

    sys.path.insert(0, os.path.join(args.ref, "scripts"))
    import pack_weights  # the reference packer, unmodified

    with tempfile.TemporaryDirectory() as td:
        snap = make_tiny_snapshot(os.path.join(td, "snap"))
        out = os.path.join(td, "out", "tiny_int8.bin")
        pack_weights.find_snapshot = lambda *a, **k: snap   # its lookup, pointed at our snapshot
        argv = sys.argv
        sys.argv = ["pack_weights.py", "--out", out]
        try:
            with redirect_stdout(io.StringIO()):
                pack_weights.main()
        finally:
            sys.argv = argv
        blob = open(out, "rb").read()
        man = json.load(open(os.path.splitext(out)[0] + ".manifest.json"))
    fx = {"blob_sha256": hashlib.sha256(blob).hexdigest(), "blob_bytes": len(blob),
          "manifest": man}
    with open(os.path.join(HERE, "pack_tiny.json"), "w") as f:
        json.dump(fx, f, indent=1)
    print("wrote pack_tiny.json:", fx["blob_sha256"], len(blob), "bytes,", len(man["tensors"]), "tensors")


if __name__ == "__main__":
    main()
