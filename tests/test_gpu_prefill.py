"""GPU parity of qwen_prefill: the prompt through every layer at once (the
DeltaNet layers by the chunked delta rule) against the golden's token-by-token
decode (golden/model.py:243-267 looped, as run_prompt.py:82-83 prefills).

Bars: W8A32 -- the last prompt token's argmax and logits (1e-4 relative) equal
to the golden's, the 64 greedy ids that follow identical to the golden's, and
the decode state after the prompt within 1e-4 (relative to each array's max)
of the state 16 single decode steps leave; chunked prompts (> 32 tokens) and a
prefill that starts from a non-empty state agree with single steps the same
way.  W8A8 -- the last prompt token's logits within 0.1 of the golden's (the
W8A8 chaos bar of the decode tests).
"""

import numpy as np
import pytest

from golden_util import LOGIT_RTOL, VOCAB, fixture, logits_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def api():
    from qwen_fpga_b200 import api as A
    return A


@pytest.fixture(scope="module")
def decs(blob_path):
    A = api()
    a = A.Decoder(blob_path, max_ctx=256)
    b = A.Decoder(blob_path, max_ctx=256)
    yield a, b
    a.close()
    b.close()


def _close(x, y, rtol=1e-4):
    scale = max(float(np.abs(y).max()), 1e-30)
    return float(np.abs(np.asarray(x) - np.asarray(y)).max()) / scale


def _states_close(ea, eb):
    errs = {"rec": _close(ea.rec, eb.rec), "conv": _close(ea.conv, eb.conv)}
    assert ea.pos == eb.pos and len(ea.kc) == len(eb.kc)
    errs["kc"] = max(_close(ea.kc[f], eb.kc[f]) for f in range(len(ea.kc)))
    errs["vc"] = max(_close(ea.vc[f], eb.vc[f]) for f in range(len(ea.vc)))
    return errs


def test_prefill_config0_matches_golden(decs):
    fx = fixture("config0.npz")
    prompt = fx["prompt"].tolist()
    pf, step = decs
    pf.reset()
    pf.set_act_int8(False)
    am, lg = pf.prefill(prompt)
    assert am == int(fx["argmax"][15])
    assert logits_close(lg, fx, "step15") < LOGIT_RTOL
    # the state equals that of 16 single decode steps
    step.reset()
    step.set_act_int8(False)
    for t in prompt:
        step.decode_step(t, want_logits=False)
    errs = _states_close(pf.export_state(), step.export_state())
    print(f"prefill vs decode state rel err {errs}")
    assert max(errs.values()) < 1e-4, errs
    # and the greedy continuation is the golden's
    ids = [am]
    for _ in range(len(fx["generated"]) - 1):
        am, _ = pf.decode_step(am, want_logits=False)
        ids.append(am)
    assert ids == fx["generated"].tolist()


@pytest.mark.parametrize("n_before,n_prompt", [(0, 40), (5, 11), (3, 70)])
def test_prefill_chunks_and_warm_start_match_steps(decs, n_before, n_prompt):
    """Prompts longer than one 32-token chunk, and a prefill after decode steps."""
    pf, step = decs
    toks = np.random.default_rng(n_before * 100 + n_prompt).integers(0, VOCAB, n_before + n_prompt).tolist()
    for d in (pf, step):
        d.reset()
        d.set_act_int8(False)
    for t in toks[:n_before]:
        pf.decode_step(t, want_logits=False)
    am_p, lg_p = pf.prefill(toks[n_before:])
    for t in toks:
        am_s, lg_s = step.decode_step(t, want_logits=True)
    assert am_p == am_s
    assert _close(lg_p, lg_s) < LOGIT_RTOL
    errs = _states_close(pf.export_state(), step.export_state())
    assert max(errs.values()) < 1e-4, errs
    # both continue identically
    a1, _ = pf.decode_step(am_p, want_logits=False)
    a2, _ = step.decode_step(am_s, want_logits=False)
    assert a1 == a2


def test_prefill_w8a8_logits(decs):
    fx = fixture("config0_w8a8.npz")
    pf, _ = decs
    pf.reset()
    pf.set_act_int8(True)
    try:
        am, lg = pf.prefill(fx["prompt"].tolist())
    finally:
        pf.set_act_int8(False)
    err = logits_close(lg, fx, "step15")
    print(f"W8A8 prefill step-15 logits rel err {err:.3e}")
    assert err < 0.1


def test_prefill_errors(decs, blob_path):
    A = api()
    pf, _ = decs
    pf.reset()
    with pytest.raises(A.QwenError) as e:
        pf.prefill([1, VOCAB])
    assert e.value.code == A.QWEN_ERR_ARG
    small = A.Decoder(blob_path, max_ctx=8)
    try:
        with pytest.raises(A.QwenError) as e:
            small.prefill(list(range(9)))
        assert e.value.code == A.QWEN_ERR_STATE
    finally:
        small.close()
