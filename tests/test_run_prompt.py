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


class _FakeTok:
    """Stands in for the snapshot's tokenizer: the chat template wraps the
    prompt's bytes in two marker ids; decode maps ids back to text."""
    eos_token_id = 2

    def __call__(self, text, return_tensors=None):
        import numpy as np

        class _E:
            input_ids = np.array([[100 + b for b in text.encode()]])
        return _E()

    def apply_chat_template(self, msgs, add_generation_prompt=True, tokenize=True):
        assert add_generation_prompt and tokenize and msgs[0]["role"] == "user"
        return {"input_ids": [7] + [100 + b for b in msgs[0]["content"].encode()] + [8]}

    def decode(self, ids):
        return "".join(f"<{i}>" for i in ids)


class _FakeDecoder:
    """Stands in for api.Decoder: the prefill's argmax and then a fixed
    continuation, recording what it was fed."""
    fed = []

    def __init__(self, blob, device=0, max_ctx=0, act_int8=False):
        self.next = iter([31, 32, 2, 33])
        _FakeDecoder.fed = []
        _FakeDecoder.act_int8 = act_int8

    def prefill(self, ids, want_logits=False):
        _FakeDecoder.fed.append(list(ids))
        return 30, None

    def decode_step(self, tok, want_logits=False):
        _FakeDecoder.fed.append(tok)
        return next(self.next), None

    def close(self):
        pass


def test_text_prompt_flow_with_a_tokenizer(monkeypatch, capsys, tmp_path):
    """With a tokenizer: the chat template (or the raw encoding) feeds the
    prefill, each generated id is fed back, printing is detokenised, and the
    tokenizer's EOS ends the answer (run_prompt.py:58-98)."""
    from qwen_fpga_b200 import api
    monkeypatch.setattr(R, "_tokenizer", lambda snap: _FakeTok())
    monkeypatch.setattr(api, "Decoder", _FakeDecoder)
    (tmp_path / "blob.bin").write_bytes(b"")
    res = R.run(["-p", "hi", "--snapshot", str(tmp_path), "--blob", str(tmp_path / "blob.bin"), "-n", "10",
                 "--w8a8"])
    assert res["prompt_ids"] == [7, 100 + ord("h"), 100 + ord("i"), 8]
    assert res["ids"] == [30, 31, 32]                    # 2 is the EOS
    assert _FakeDecoder.fed == [res["prompt_ids"], 30, 31, 32] and _FakeDecoder.act_int8
    assert "<30><31><32>" in capsys.readouterr().out.replace(" ", "")
    res = R.run(["-p", "hi", "--raw", "--snapshot", str(tmp_path), "--blob", str(tmp_path / "blob.bin"), "-n", "2"])
    assert res["prompt_ids"] == [100 + ord("h"), 100 + ord("i")] and res["ids"] == [30, 31]
