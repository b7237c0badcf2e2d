"""W8A8 (ACT_INT8) arithmetic inside the persistent decode step, pinned bit
for bit.

The whole-step W8A8 tests can only bound agreement statistically (one-ulp
differences flip rint decisions and the flips persist), so this file pins the
integer arithmetic itself.  For one GEMV phase of a real step the kernel
records (qwen_capture_phase / qwen_capture_read) its fp32 input, the int8
activations and s_x it quantised them to, and the int32 accumulator of every
output row.  The test recomputes on the CPU:
  * the input of a normed phase (IN, GATEUP) from the kernel's residual h with
    the golden RMSNorm (golden/model.py:63-75, the oracle's norm_1pw);
  * the golden per-vector quantiser _qa (golden/model.py:37-45, the oracle's
    act_int8) of that input: x_q and s_x must be bit-identical;
  * acc = q_w @ x_q in int64 (scripts/export_gemv_tv.py:49): every row must
    be identical.
Phases: IN, OUT, GATEUP and DOWN of a DeltaNet layer, IN and OUT of an
attention layer.
"""

import numpy as np
import pytest

from oracle import golden_port as P

pytestmark = pytest.mark.gpu

PROMPT = [9001, 123456, 77, 248000]


def phase_rows(blob, p):
    """int8 weight rows of GEMV phase p in the kernel's row order."""
    l, sub = divmod(p, 5)
    pre = f"layers.{l}."
    linear = l % 4 != 3
    if sub == 0:
        names = ([pre + "linear_attn.in_proj_qkv.weight", pre + "linear_attn.in_proj_z.weight"] if linear else
                 [pre + "self_attn.q_proj.weight", pre + "self_attn.k_proj.weight", pre + "self_attn.v_proj.weight"])
    elif sub == 2:
        names = [pre + ("linear_attn.out_proj.weight" if linear else "self_attn.o_proj.weight")]
    elif sub == 3:
        names = [pre + "mlp.gate_proj.weight", pre + "mlp.up_proj.weight"]
    else:
        names = [pre + "mlp.down_proj.weight"]
    return np.concatenate([blob.int8(n)[0] for n in names], axis=0)


@pytest.fixture(scope="module")
def dec(blob_path):
    from qwen_fpga_b200 import api
    d = api.Decoder(blob_path, max_ctx=64)
    d.set_act_int8(True)
    yield d
    d.close()


@pytest.mark.parametrize("phase", [5, 7, 8, 9, 15, 17])
def test_w8a8_phase_arithmetic_is_exact(dec, blob, cfg, phase):
    dec.reset()
    for t in PROMPT[:3]:
        dec.decode_step(t, want_logits=False)
    dec.capture_phase(phase)
    try:
        dec.decode_step(PROMPT[3], want_logits=False)
        cap = dec.capture_read()
    finally:
        dec.capture_phase(-1)
    assert cap["captured"]
    l, sub = divmod(phase, 5)
    x = cap["x"]
    if sub in (0, 3):
        w = blob.fp32(f"layers.{l}." + ("input_layernorm.weight" if sub == 0 else "post_attention_layernorm.weight"))
        x = P.norm_1pw(x.astype(np.float32), w, np.float32(cfg["rms_norm_eps"])).astype(np.float32)
    xq, sx = P.act_int8(x)
    assert cap["sx"] == sx, (float(cap["sx"]), float(sx))
    assert np.array_equal(cap["xq"], xq), int(np.sum(cap["xq"] != xq))
    rows = phase_rows(blob, phase)
    assert rows.shape[1] == cap["K"]
    acc = rows.astype(np.int64) @ xq.astype(np.int64)
    assert np.array_equal(cap["acc"][:rows.shape[0]].astype(np.int64), acc)
