"""The prompt front-end on the GPU: the config-0 prompt as token ids through
`python -m qwen_fpga_b200.run_prompt --synthetic` (one qwen_prefill, then
qwen_decode_step per token) generates the reference golden's 64 tokens."""

import json
import os
import subprocess
import sys

import pytest

from golden_util import fixture

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_run_prompt_ids_match_golden(blob_path):
    fx = fixture("config0.npz")
    from qwen_fpga_b200 import run_prompt as R
    res = R.run(["--synthetic", "--ids", ",".join(str(int(t)) for t in fx["prompt"]), "-n", "64", "--quiet"])
    assert res["ids"] == [int(t) for t in fx["generated"]]
    assert res["prompt_ids"] == [int(t) for t in fx["prompt"]]


def test_run_prompt_cli_eos_stops(blob_path):
    """As a command: an EOS id given with --eos ends the answer before it."""
    fx = fixture("config0.npz")
    ids = ",".join(str(int(t)) for t in fx["prompt"])
    stop = int(fx["generated"][5])
    out = subprocess.run([sys.executable, "-m", "qwen_fpga_b200.run_prompt", "--synthetic", "--ids", ids,
                          "-n", "64", "--eos", str(stop), "--quiet"], cwd=REPO, capture_output=True, text=True,
                         check=True)
    res = json.loads(out.stdout.strip().splitlines()[-1])
    assert res["ids"] == [int(t) for t in fx["generated"][:5]]
