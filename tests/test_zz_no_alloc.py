"""The allocation-free GEMV + argmax entry point (qwen_gemv_i8_f32_argmax_noalloc).

Collected last on purpose.  It runs after every other test has used the library
in the same process, so it also checks that the static scratch starts each call
re-armed.

GPU: y equals what the existing qwen_gemv_i8_f32 returns for the same inputs,
and argmax is the first index of the largest y (np.argmax, the head rule of
golden/model.py:266-267).  This holds on two calls in a row and on shapes that
leave a ragged last block.  Calls after the first allocate nothing (the
device's free memory is unchanged across them).  CPU: sizes beyond the static
scratch are rejected before any device work.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def api():
    from qwen_fpga_b200 import api as A
    return A


def inputs(N, K, seed):
    rng = np.random.default_rng(seed)
    w = rng.integers(-127, 128, (N, K), dtype=np.int8)
    s = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    return w, s, x


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("N,K", [(248320, 1024), (6144, 1024), (1000, 3584), (1, 32)])
def test_noalloc_argmax_matches_gemv_twice(N, K):
    A = api()
    w, s, x = inputs(N, K, seed=N + K)
    dw, ds = dev(w), dev(s)
    am = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    for call, xv in enumerate((x, -0.5 * x[::-1].copy())):   # two calls in a row, different x
        dx = dev(xv)
        y_ref = A.gemv_i8_f32(dw, ds, dx)
        y = torch.empty(N, dtype=torch.float32, device="cuda")
        A.gemv_i8_f32_argmax_noalloc(dw, ds, dx, am, y=y)
        torch.cuda.synchronize()
        y_ref = y_ref.cpu().numpy()
        y = y.cpu().numpy()
        # same arithmetic as the existing entry point: bit-identical in practice, bar 1e-6
        assert np.abs(y - y_ref).max() <= 1e-6 * max(np.abs(y_ref).max(), 1e-30), call
        assert int(am.item()) == int(np.argmax(y_ref)), call


@pytest.mark.gpu
def test_noalloc_call_allocates_nothing():
    """After the first call on the device (which resolves the static array's
    address and may load the library's device code), calls leave the device's
    free memory unchanged: nothing is allocated per call."""
    A = api()
    N, K = 6144, 1024
    w, s, x = inputs(N, K, seed=5)
    dw, ds, dx = dev(w), dev(s), dev(x)
    y = torch.empty(N, dtype=torch.float32, device="cuda")
    am = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    A.gemv_i8_f32_argmax_noalloc(dw, ds, dx, am, y=y)      # first call: set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        A.gemv_i8_f32_argmax_noalloc(dw, ds, dx, am, y=y)
        A.gemv_i8_f32_argmax_noalloc(dw, ds, dx, am)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    assert int(am.item()) == int(np.argmax(y.cpu().numpy()))


@pytest.mark.gpu
def test_noalloc_argmax_signed_zero_and_nan():
    """np.argmax rules: -0.0 and +0.0 are equal (the first index wins), and the
    first NaN wins over every number."""
    A = api()
    N, K = 3000, 32
    w = np.zeros((N, K), np.int8)
    w[:, 0] = -1
    w[[5, 2900], 0] = 0                # rows 5 and 2900 give exactly 0.0 ...
    s = np.full(N, 0.01, np.float32)
    s[5] = -0.01                       # ... row 5 as -0.0 (0 * negative scale)
    x = np.zeros(K, np.float32)
    x[0] = 1.0
    am = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    y = torch.empty(N, dtype=torch.float32, device="cuda")
    A.gemv_i8_f32_argmax_noalloc(dev(w), dev(s), dev(x), am, y=y)
    torch.cuda.synchronize()
    yh = y.cpu().numpy()
    assert np.signbit(yh[5]) and yh[5] == 0.0 and not np.signbit(yh[2900])
    assert int(am.item()) == int(np.argmax(yh)) == 5
    s2 = s.copy()
    s2[[700, 1200]] = np.nan           # NaN rows: the first one is the argmax
    A.gemv_i8_f32_argmax_noalloc(dev(w), dev(s2), dev(x), am, y=y)
    torch.cuda.synchronize()
    assert int(am.item()) == int(np.argmax(y.cpu().numpy())) == 700


@pytest.mark.gpu
def test_noalloc_argmax_without_y_and_ties():
    """y may be NULL; equal maxima resolve to the first index."""
    A = api()
    N, K = 5000, 64
    w = np.zeros((N, K), np.int8)
    w[[17, 4001, 4999], :] = 3        # three identical best rows
    s = np.full(N, 0.01, np.float32)
    x = np.ones(K, np.float32)
    am = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    for _ in range(2):
        A.gemv_i8_f32_argmax_noalloc(dev(w), dev(s), dev(x), am)
        torch.cuda.synchronize()
        assert int(am.item()) == 17


def test_noalloc_rejects_sizes_beyond_scratch():
    """N above the 1,048,576 rows the static scratch covers is refused before any launch."""
    from qwen_fpga_b200 import api as A
    import ctypes as C
    L = A.load()
    buf = C.create_string_buffer(64)
    p = C.cast(buf, C.c_void_p)
    with pytest.raises(A.QwenError) as ei:
        A._check(L.qwen_gemv_i8_f32_argmax_noalloc(p, p, p, p, p, 1048577, 1024, None))
    assert ei.value.code == 1 and "1048576" in str(ei.value)
