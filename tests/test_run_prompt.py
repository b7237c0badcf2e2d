"""The prompt front-end (qwen_fpga_b200.run_prompt, the counterpart of the
reference's run_prompt.py): argument handling on the CPU; the GPU run is in
test_gpu_prompt.py."""

import pytest

from qwen_fpga_b200 import run_prompt as R


def test_parse_ids():
    assert R.parse_ids("1,2, 3") == [1, 2, 3]
    assert R.parse_ids("7,") == [7]
    with pytest.raises(ValueError):
        R.parse_ids(",")
    with pytest.raises(ValueError):
        R.parse_ids("1,x")


def test_prompt_source_is_required_and_exclusive():
    with pytest.raises(SystemExit):
        R.build_parser().parse_args(["-n", "4"])
    with pytest.raises(SystemExit):
        R.build_parser().parse_args(["-p", "hi", "--ids", "1,2"])
    a = R.build_parser().parse_args(["--ids", "1,2", "--synthetic", "--w8a8", "--eos", "5", "--eos", "6"])
    assert a.ids == "1,2" and a.synthetic and a.w8a8 and a.eos == [5, 6] and a.n_new == 64


def test_text_prompt_without_tokenizer_is_refused():
    with pytest.raises(SystemExit, match="needs a tokenizer"):
        R.run(["-p", "hello", "--synthetic"])


def test_ids_without_weights_is_refused():
    with pytest.raises(SystemExit, match="--blob"):
        R.run(["--ids", "1,2"])
    with pytest.raises(SystemExit, match="no --snapshot"):
        R.run(["--ids", "1,2", "--blob", "/nonexistent/qwen.bin"])
