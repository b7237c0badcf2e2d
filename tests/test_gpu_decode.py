"""GPU parity of the whole decode step through the C ABI (qwen_decode_step /
qwen_generate) against the reference golden model's committed vectors and the
oracle port.

Bar: identical greedy token ids; fp32 logits within 1e-4 of the golden's,
relative to the golden's max |logit| (golden_util.LOGIT_RTOL).
"""

import numpy as np
import pytest

from golden_util import LOGIT_RTOL, fixture, logits_close
from qwen_fpga_b200.api import VOCAB
from oracle import golden_port as P

pytestmark = pytest.mark.gpu

MAX_CTX = 32768 + 64


@pytest.fixture(scope="module")
def dec(blob_path):
    """One context (the persistent decode kernel) shared by the tests."""
    from qwen_fpga_b200 import api
    d = api.Decoder(blob_path, max_ctx=MAX_CTX)
    yield d
    d.close()


def test_config0_generate_matches_golden(dec):
    fx = fixture("config0.npz")
    dec.reset()
    dec.set_act_int8(False)
    ids, sec = dec.generate(fx["prompt"].tolist(), 64)
    assert ids == fx["generated"].tolist()
    assert sec > 0


def test_config0_step_logits_match_golden(dec):
    """decode_step with logits: every step's argmax and the stored logits."""
    fx = fixture("config0.npz")
    dec.reset()
    dec.set_act_int8(False)
    feed = fx["prompt"].tolist() + fx["generated"].tolist()
    errs = {}
    for i, t in enumerate(feed):
        want = i in (0, 15, 79)
        am, lg = dec.decode_step(t, want_logits=want)
        assert am == int(fx["argmax"][i]), f"step {i}"
        if want:
            errs[i] = logits_close(lg, fx, f"step{i}")
    assert max(errs.values()) < LOGIT_RTOL, errs


def test_pinned_logits_written_by_the_kernel_match_the_copy(dec):
    """Page-locked host logits are written by the head kernel itself; pageable
    ones are copied after it.  Both give the same logits bit for bit, every
    step, and the golden's at step 15."""
    import torch
    fx = fixture("config0.npz")
    pinned = torch.empty(VOCAB, dtype=torch.float32, pin_memory=True).numpy()
    runs = []
    for buf in (pinned, np.empty(VOCAB, np.float32)):
        dec.reset()
        dec.set_act_int8(False)
        got = []
        for t in fx["prompt"].tolist():
            am, lg = dec.decode_step(t, want_logits=True, out=buf)
            got.append((am, lg.copy()))
        runs.append(got)
    for (a0, l0), (a1, l1) in zip(*runs):
        assert a0 == a1 and np.array_equal(l0, l1)
    assert logits_close(runs[0][15][1], fx, "step15") < LOGIT_RTOL


def test_generate_and_step_paths_agree(dec):
    fx = fixture("config0.npz")
    prompt = fx["prompt"].tolist()[:5]
    dec.reset()
    ids_g, _ = dec.generate(prompt, 6)
    dec.reset()
    am = None
    for t in prompt:
        am, _ = dec.decode_step(t, want_logits=False)
    ids_s = []
    for _ in range(6):
        ids_s.append(am)
        am, _ = dec.decode_step(am, want_logits=False)
    assert ids_g == ids_s


def test_config0_w8a8_teacher_forced_matches_golden(dec):
    """ACT_INT8 (W8A8) from a cold state, fed the golden's own token stream.

    W8A8 re-quantises every projection input with rint, so a one-ulp difference
    anywhere can flip an int8 activation digit, and the flip persists in the
    DeltaNet state.  The unmodified golden, fed the same tokens with 1e-7..3e-6
    relative noise on three weight tensors, agrees with itself on 58-74 of the
    80 argmaxes (fixture key self_agreement).  Bar: agreement within that spread
    (>= its minimum - 2), and step-0 logits within 0.1: the exact-integer GEMVs
    differ from the golden's BLAS sums by ~1e-7 relative, which already flips a
    handful of rint decisions per step (each flip moves the logits by ~1e-2)."""
    fx = fixture("config0_w8a8.npz")
    floor = int(fx["self_agreement"].min()) - 2
    feed = fx["prompt"].tolist() + fx["generated"].tolist()
    dec.reset()
    dec.set_act_int8(True)
    try:
        agree = 0
        errs = {}
        for i, t in enumerate(feed):
            want = i in (0, 15, 79)
            am, lg = dec.decode_step(t, want_logits=want)
            agree += int(am == int(fx["argmax"][i]))
            if want:
                errs[i] = logits_close(lg, fx, f"step{i}")
    finally:
        dec.set_act_int8(False)
    print(f"W8A8 teacher-forced agreement {agree}/80 (golden self-agreement "
          f"{fx['self_agreement'].tolist()}), logits rel err {errs}")
    assert agree >= floor
    assert errs[0] < 0.1


def test_config2_w8a8_warm_step_matches_golden(dec, cfg):
    """ACT_INT8 warm start (rec N(0,0.1), 4096 cached positions N(0,1)), six
    greedy steps fed back as the golden feeds them.

    This start is chaotic: the golden's own step-0 logits move by 1.75e-2
    (relative to max |logit|) when its warm state is perturbed by 3e-7 relative
    (fixture key step0_sens_3e-07).  Bar: all six argmaxes identical to the
    golden's, and the step-0 and step-5 logits within 0.1 (measured on B200:
    4.9e-2 and 5.8e-2).  The integer arithmetic under this chaos is pinned
    bit-exactly by tests/test_gpu_w8a8_capture.py."""
    fx = fixture("config2.npz")
    assert float(fx["step0_sens_3e-07"]) > 1e-3
    st = P.warm_state(cfg, int(fx["T0"]), seed=2)
    dec.reset()
    dec.set_act_int8(True)
    errs = {}
    try:
        dec.import_state(st)
        tok = int(fx["first_token"])
        for j in range(len(fx["argmax"])):
            am, lg = dec.decode_step(tok, want_logits=True)
            assert am == int(fx["argmax"][j]), f"step {j}"
            if f"step{j}_sample" in fx.files:
                errs[j] = logits_close(lg, fx, f"step{j}")
            tok = am
    finally:
        dec.set_act_int8(False)
    print(f"W8A8 warm logits rel err {errs}")
    assert sorted(errs) == [0, 5]
    assert max(errs.values()) < 0.1


def test_config3_long_context_matches_golden(dec, cfg):
    fx = fixture("config3.npz")
    st = P.warm_state(cfg, int(fx["T0"]), seed=3)
    dec.reset()
    dec.import_state(st)
    del st
    tok = int(fx["first_token"])
    for j in range(len(fx["argmax"])):
        am, lg = dec.decode_step(tok, want_logits=True)
        assert am == int(fx["argmax"][j])
        assert logits_close(lg, fx, f"step{j}") < LOGIT_RTOL
        tok = am


def test_state_roundtrip_and_port_agreement(dec, cfg, fq_weights):
    """After 6 steps the exported state matches the port's state, and a
    re-import continues bit-identically."""
    fx = fixture("config0.npz")
    toks = fx["prompt"].tolist()[:6]
    dec.reset()
    for t in toks:
        dec.decode_step(t, want_logits=False)
    ex = dec.export_state()
    assert ex.pos == 6 and len(ex.kc) == 6 and ex.kc[0].shape == (6, 2, 256)
    port = P.PortDecoder(fq_weights, cfg)
    pst = P.PortState.zeros(cfg)
    for t in toks:
        port.step(t, pst)
    scale = np.abs(pst.rec).max()
    assert np.abs(ex.rec - pst.rec).max() < 1e-4 * scale
    assert np.abs(ex.conv - pst.conv).max() < 1e-4 * np.abs(pst.conv).max()
    for f in range(6):
        assert np.abs(ex.kc[f] - pst.kc[f]).max() < 1e-4 * np.abs(pst.kc[f]).max()
        assert np.abs(ex.vc[f] - pst.vc[f]).max() < 1e-4 * np.abs(pst.vc[f]).max()
    am1, lg1 = dec.decode_step(123, want_logits=True)
    dec.reset()
    dec.import_state(ex)
    am2, lg2 = dec.decode_step(123, want_logits=True)
    assert am1 == am2 and np.array_equal(lg1, lg2)


def test_matches_reference_hls_decoder(dec, blob_path):
    """Second oracle: the reference's own HLS C++ qwen_top on the same blob."""
    from oracle import native
    if not native.have_ref():
        pytest.skip("oracle/_ref not built")
    fx = fixture("config0.npz")
    ref = native.HlsRef(blob_path)
    dec.reset()
    for t in fx["prompt"].tolist()[:3]:
        am_r, lg_r = ref.step(t, want_logits=True)
        am_g, lg_g = dec.decode_step(t, want_logits=True)
        assert am_r == am_g
        assert np.abs(lg_r - lg_g).max() < LOGIT_RTOL * np.abs(lg_r).max()
    ref.close()


def test_errors_are_reported(dec):
    from qwen_fpga_b200 import api
    with pytest.raises(api.QwenError) as e:
        dec.decode_step(248320)
    assert e.value.code == api.QWEN_ERR_ARG
    with pytest.raises(api.QwenError):
        dec.decode_step(-1)
    small = api.Decoder(dec_blob_path(dec), max_ctx=4)
    try:
        for t in range(4):
            small.decode_step(t, want_logits=False)
        with pytest.raises(api.QwenError) as e:
            small.decode_step(5, want_logits=False)
        assert e.value.code == api.QWEN_ERR_STATE
        with pytest.raises(api.QwenError):
            small.generate([1, 2, 3], 5)
    finally:
        small.close()


def dec_blob_path(dec):
    from qwen_fpga_b200 import synth
    return synth.ensure_blob(1234)
