"""GPU parity of the standalone GEMV and delta-rule operators (C ABI).

* int8 x int8: accumulators bit-exact against the reference's int32 product
  (scripts/export_gemv_tv.py:49) on every config-1 shape, and the dequantised
  y bit-exact against export_gemv_tv.py:50.
* int8 x fp32: bit-exact against a numpy restatement of the kernel's own
  fixed-point digit algorithm, and within 2e-6 (relative to max |y|) of an
  fp64 product -- the fp32 contract of hls/src/gemv.hpp:28-42.
* delta rule: within 2e-5 absolute of the golden's traced layer
  (the bar of hls/tb/tb_deltanet.cpp:91).
"""

import zlib

import numpy as np
import pytest

from golden_util import fixture
from oracle import golden_port as P
from test_oracle import GEMV_SHAPES, gemv_inputs

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def api():
    from qwen_fpga_b200 import api as A
    return A


def digits_reference(w, s, x):
    """numpy restatement of the W8A32 digit GEMV (bit-exact target of the kernel)."""
    x = x.astype(np.float32)
    amax = np.float32(np.abs(x).max())
    if amax == 0:
        return np.zeros(w.shape[0], np.float32)
    _, e = np.frexp(amax)
    sh = 22 - int(e)
    X = np.rint(np.ldexp(x, sh)).astype(np.int64)
    Y = w.astype(np.int64) @ X
    return ((Y.astype(np.float64) * 2.0 ** -sh) * s.astype(np.float64)).astype(np.float32)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("N,K", GEMV_SHAPES)
def test_gemv_i8_i8_bit_exact(N, K):
    fx = fixture("gemv_i8.npz")
    w, sw, x, sx = gemv_inputs(N, K)
    acc, y = api().gemv_i8_i8(dev(w), dev(sw), dev(x), sx)
    torch.cuda.synchronize()
    acc = acc.cpu().numpy()
    y = y.cpu().numpy()
    key = f"{N}x{K}"
    assert zlib.crc32(acc.tobytes()) == int(fx[key + "_crc"])
    ref = P.gemv_int32(w, x)
    assert np.array_equal(acc, ref)
    assert np.array_equal(y, P.gemv_dequant(ref, sx, sw))


def test_gemv_i8_i8_real_activation(blob):
    fx = fixture("w8a8_gemv.npz")
    wq, ws = blob.int8("layers.3.self_attn.k_proj.weight")
    acc, y = api().gemv_i8_i8(dev(wq), dev(ws), dev(fx["x_i8"]), float(fx["sx"]))
    torch.cuda.synchronize()
    assert np.array_equal(acc.cpu().numpy(), fx["acc"])
    assert np.array_equal(y.cpu().numpy(), fx["y"])


@pytest.mark.parametrize("N,K", GEMV_SHAPES + [(1, 32), (3, 1024), (1000, 2048), (7, 3584)])
def test_gemv_i8_f32(N, K):
    rng = np.random.default_rng(N * 7 + K)
    w = rng.integers(-127, 128, (N, K), dtype=np.int8)
    s = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    y = api().gemv_i8_f32(dev(w), dev(s), dev(x))
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    assert np.array_equal(y, digits_reference(w, s, x))
    ref = (w.astype(np.float64) @ x.astype(np.float64)) * s.astype(np.float64)
    assert np.abs(y - ref).max() <= 2e-6 * np.abs(ref).max()


def test_gemv_i8_f32_zero_and_tiny_inputs():
    rng = np.random.default_rng(5)
    w = rng.integers(-127, 128, (64, 256), dtype=np.int8)
    s = np.ones(64, np.float32)
    y = api().gemv_i8_f32(dev(w), dev(s), dev(np.zeros(256, np.float32)))
    torch.cuda.synchronize()
    assert (y.cpu().numpy() == 0).all()
    x = (rng.standard_normal(256) * 1e-20).astype(np.float32)
    y = api().gemv_i8_f32(dev(w), dev(s), dev(x))
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy(), digits_reference(w, s, x))


def test_gemv_rejects_bad_shapes():
    A = api()
    w = torch.zeros((4, 48), dtype=torch.int8, device="cuda")
    s = torch.ones(4, device="cuda")
    x = torch.ones(48, device="cuda")
    with pytest.raises(A.QwenError) as e:
        A.gemv_i8_f32(w, s, x)
    assert e.value.code == A.QWEN_ERR_ARG
    w2 = torch.zeros((4, 4096), dtype=torch.int8, device="cuda")
    with pytest.raises(A.QwenError):
        A.gemv_i8_f32(w2, s, torch.ones(4096, device="cuda"))


def test_delta_rule_matches_golden_trace():
    fx = fixture("deltanet_trace.npz")
    rng = np.random.default_rng(11)
    S = (rng.standard_normal((16, 128, 128)) * 0.05).astype(np.float32)
    heads = fx["heads"]
    S[heads] = fx["S_in"]
    Sd = dev(S)
    out = api().delta_rule_layer(dev(fx["q"]), dev(fx["k"]), dev(fx["v"]), dev(fx["g"]),
                                 dev(fx["beta"]), Sd)
    torch.cuda.synchronize()
    out = out.cpu().numpy()
    S2 = Sd.cpu().numpy()
    # the reference heads against the golden trace, tol of hls/tb/tb_deltanet.cpp:91
    assert np.abs(out[heads] - fx["o_core"][heads]).max() < 2e-5
    assert np.abs(S2[heads] - fx["S_out"]).max() < 2e-5
    # every head against the port's delta rule on the same state
    Sr = S.copy()
    Sr *= np.exp(fx["g"])[:, None, None]
    kv = np.einsum("hkv,hk->hv", Sr, fx["k"])
    d = (fx["v"] - kv) * fx["beta"][:, None]
    Sr += np.einsum("hk,hv->hkv", fx["k"], d)
    o = np.einsum("hkv,hk->hv", Sr, fx["q"])
    assert np.abs(S2 - Sr).max() < 2e-5
    assert np.abs(out - o).max() < 2e-5
