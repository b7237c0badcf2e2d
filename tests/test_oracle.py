"""CPU tests: the oracle and the packer against vectors the reference produced.

The fixtures under tests/golden/ were written by tests/golden/make_golden.py,
which ran the unmodified reference golden model (golden/model.py,
golden/quant.py, scripts/export_gemv_tv.py) in the build container.
"""

import json
import os
import zlib

import numpy as np
import pytest

from golden_util import SAMPLE_IDX, fixture, logits_close
from oracle import golden_port as P
from oracle import native
from qwen_fpga_b200 import synth

HERE = os.path.dirname(os.path.abspath(__file__))
GEMV_SHAPES = [(6144, 1024), (2048, 1024), (7168, 1024), (1024, 3584), (1024, 2048),
               (4096, 1024), (248320, 1024)]


def gemv_inputs(N, K, seed=0):
    rng = np.random.default_rng(seed)
    w = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sw = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    x = rng.integers(-127, 128, K, dtype=np.int8)
    sx = np.float32(rng.uniform(1e-3, 1e-2))
    return w, sw, x, sx


def test_layout_matches_reference_manifest():
    """Offsets, sizes and the flat index equal the reference's own
    artifacts/qwen35_int8.manifest.json and artifacts/weights.idx."""
    ref = json.load(open(os.path.join(HERE, "golden", "ref_layout.json")))
    man = synth.layout(synth.model_config())
    assert man["total_bytes"] == ref["total_bytes"] == 758618112
    assert man["config"] == ref["config"]
    got = [[t["name"], t["offset"], t["nbytes"], t.get("scale_offset", 0), t["dtype"]]
           for t in man["tensors"]]
    assert got == ref["tensors"]
    assert synth.index_lines(man) == ref["idx_lines"]


def test_quantize_rows_edge_cases():
    w = np.array([[0.0, 0.0, 0.0], [1.0, -2.0, 0.5], [-1e-30, 0.0, 1e-30]], np.float32)
    q, s = synth.quantize_rows(w)
    assert s[0] == 1.0 and (q[0] == 0).all()          # all-zero row: scale 1
    assert q[1].tolist() == [64, -127, 32] and s[1] == np.float32(2.0) / np.float32(127.0)
    assert np.abs(q).max() <= 127


def test_blob_is_the_pinned_random_init(blob):
    fx = fixture("config0.npz")
    assert blob.digest() == str(fx["blob_sha256"])


@pytest.mark.slow
def test_port_config0_matches_golden(fq_weights, cfg):
    """80 calls of the port (16 prompt tokens + 64 greedy) reproduce the golden's
    argmax stream and logits (config 0)."""
    fx = fixture("config0.npz")
    dec = P.PortDecoder(fq_weights, cfg)
    st = P.PortState.zeros(cfg)
    logits = None
    argmax = []
    for i, t in enumerate(fx["prompt"]):
        logits = dec.step(int(t), st)
        argmax.append(int(np.argmax(logits)))
        if i in (0, 15):
            assert logits_close(logits, fx, f"step{i}") < 1e-6
    gen = []
    for _ in range(64):
        nxt = int(np.argmax(logits))
        gen.append(nxt)
        logits = dec.step(nxt, st)
        argmax.append(int(np.argmax(logits)))
    assert logits_close(logits, fx, "step79") < 1e-6
    assert gen == fx["generated"].tolist()
    assert argmax == fx["argmax"].tolist()


@pytest.mark.slow
def test_port_config2_w8a8_matches_golden(fq_weights, cfg):
    fx = fixture("config2.npz")
    dec = P.PortDecoder(fq_weights, cfg, act_int8=True)
    st = P.warm_state(cfg, int(fx["T0"]), seed=2)
    tok = int(fx["first_token"])
    got = []
    for j in range(len(fx["argmax"])):
        lg = dec.step(tok, st)
        tok = int(np.argmax(lg))
        got.append(tok)
        if f"step{j}_sample" in fx:
            assert logits_close(lg, fx, f"step{j}") < 1e-6
    assert got == fx["argmax"].tolist()


def test_port_delta_rule_matches_trace(fq_weights, cfg):
    """Warm 5 tokens, trace linear layer 0 on the 6th (scripts/export_testvectors.py:31-40)."""
    fx = fixture("deltanet_trace.npz")
    c0 = fixture("config0.npz")
    dec = P.PortDecoder(fq_weights, cfg)
    st = P.PortState.zeros(cfg)
    for t in c0["prompt"][:5]:
        dec.step(int(t), st)
    dec.trace = {"layer": 0}
    dec.step(int(c0["prompt"][5]), st)
    tr = dec.trace
    for k in ("q", "k", "v", "g", "beta", "o_core"):
        np.testing.assert_allclose(tr[k], fx[k], rtol=0, atol=1e-6)
    h = fx["heads"]
    np.testing.assert_allclose(tr["S_in"][h], fx["S_in"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(tr["S_out"][h], fx["S_out"], rtol=0, atol=1e-6)


@pytest.mark.parametrize("N,K", GEMV_SHAPES)
def test_gemv_int32_oracles_match_reference_digests(N, K):
    """numpy int32 product and the C port give the reference's accumulators exactly."""
    fx = fixture("gemv_i8.npz")
    w, sw, x, sx = gemv_inputs(N, K)
    acc = P.gemv_int32(w, x)
    key = f"{N}x{K}"
    assert zlib.crc32(acc.tobytes()) == int(fx[key + "_crc"])
    assert int(acc.astype(np.int64).sum()) == int(fx[key + "_sum"])
    assert np.array_equal(acc[:32], fx[key + "_head"])
    y = P.gemv_dequant(acc, sx, sw)
    assert np.array_equal(y[:32], fx[key + "_yhead"])
    if N <= 8192:
        acc2, y2 = native.gemv_i8_i8(w, sw, x, sx, threads=4)
        assert np.array_equal(acc2, acc)
        assert np.array_equal(y2, y)


def test_act_quantiser_matches_reference_vector(blob):
    """export_gemv_tv.q_i8_vec on a real activation, and its int32 product."""
    fx = fixture("w8a8_gemv.npz")
    q, s = P.act_int8(fx["hn"])
    assert np.array_equal(q, fx["x_i8"]) and s == fx["sx"]
    wq, ws = blob.int8("layers.3.self_attn.k_proj.weight")
    acc = P.gemv_int32(wq, q)
    assert np.array_equal(acc, fx["acc"])
    assert np.array_equal(P.gemv_dequant(acc, s, ws), fx["y"])


def test_act_roundtrip_edge_cases():
    z = np.zeros(8, np.float32)
    assert P.act_roundtrip(z, True) is z                     # all-zero vector passes through
    x = np.array([0.5, -1.0, 0.25, 1e-9], np.float32)
    r = P.act_roundtrip(x, True)
    assert r[1] == np.float32(-1.0) and abs(r[3]) == 0.0
    assert P.act_roundtrip(x, False) is x


@pytest.mark.slow
def test_hls_reference_matches_golden_first_steps(blob_path):
    """The reference's own HLS C++ decoder (built into oracle/_ref) on the same
    blob: argmax equal to the golden's for the first 4 prompt steps and step-0
    logits within the reference's own tb_decode bar (hls/tb/tb_decode.cpp:112)."""
    if not native.have_ref():
        pytest.skip("oracle/_ref not built (needs the reference checkout)")
    fx = fixture("config0.npz")
    ref = native.HlsRef(blob_path)
    for i in range(4):
        am, lg = ref.step(int(fx["prompt"][i]), want_logits=(i == 0))
        assert am == int(fx["argmax"][i])
        if i == 0:
            assert np.abs(lg[SAMPLE_IDX] - fx["step0_sample"]).max() < 5e-2
            assert logits_close(lg, fx, "step0") < 1e-4
    ref.close()


def test_synth_warm_state_matches_port_recipe(cfg):
    """bench.py draws the config 2/3 warm starts with synth.warm_state_arrays
    (the product side may not import the oracle); it must be the recipe the
    parity fixtures were generated with (oracle golden_port.warm_state)."""
    from qwen_fpga_b200 import synth
    a = synth.warm_state_arrays(7, seed=2)
    b = P.warm_state(cfg, 7, seed=2)
    assert a.pos == b.pos == 7
    assert np.array_equal(a.rec, b.rec) and np.array_equal(a.conv, b.conv)
    for f in range(6):
        assert np.array_equal(a.kc[f], b.kc[f]) and np.array_equal(a.vc[f], b.vc[f])


@pytest.mark.parametrize("n", [1, 2, 7, 16, 32])
def test_chunked_delta_rule_equals_recurrence(n):
    """The chunked (WY) delta rule of the GPU prefill against the golden's
    recurrence on random unit-norm q/k, decays in [-1, 0) and gates in (0, 1),
    from a warm state."""
    rng = np.random.default_rng(n)
    K = V = 128
    S = (rng.standard_normal((K, V)) * 0.1).astype(np.float32)
    q = rng.standard_normal((n, K)).astype(np.float32)
    k = rng.standard_normal((n, K)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    k /= np.linalg.norm(k, axis=1, keepdims=True)
    q *= np.float32(K ** -0.5)
    v = rng.standard_normal((n, V)).astype(np.float32)
    g = -rng.uniform(0.0, 1.0, n).astype(np.float32)
    beta = rng.uniform(0.05, 0.95, n).astype(np.float32)
    o_r, S_r = P.delta_rule_steps(S, q, k, v, g, beta)
    o_c, S_c = P.delta_rule_chunk(S, q, k, v, g, beta)
    assert np.abs(o_c - o_r).max() < 1e-5 * np.abs(o_r).max()
    assert np.abs(S_c - S_r).max() < 1e-5 * np.abs(S_r).max()


def test_chunked_delta_rule_reproduces_the_golden_trace():
    """One token of the chunked form reproduces the golden's traced layer-0
    delta rule (heads 0 and 9 of deltanet_trace.npz)."""
    fx = fixture("deltanet_trace.npz")
    for i, h in enumerate(fx["heads"]):
        o, S2 = P.delta_rule_chunk(fx["S_in"][i], fx["q"][h][None], fx["k"][h][None], fx["v"][h][None],
                                   fx["g"][h:h + 1], fx["beta"][h:h + 1])
        np.testing.assert_allclose(o[0], fx["o_core"][h], rtol=0, atol=2e-6)
        np.testing.assert_allclose(S2, fx["S_out"][i], rtol=0, atol=2e-6)


@pytest.mark.parametrize("Tn,n_slices,n_chunks", [(1, 2, 64), (1, 4, 64), (3, 4, 64), (17, 2, 64), (80, 4, 5),
                                                  (1000, 1, 64), (1000, 2, 64), (4097, 4, 64)])
def test_split_kv_combine_equals_softmax_attention(Tn, n_slices, n_chunks):
    """The decode kernel's split of a KV group's positions into rank slices and
    chunks, merged by (m, l, o) in order with empty slices skipped (the case
    Tn < ranks of the group), is the golden's softmax attention
    (golden/model.py:219-229) up to rounding."""
    rng = np.random.default_rng(Tn * 10 + n_slices)
    q = rng.standard_normal((4, 256)).astype(np.float32)
    K = rng.standard_normal((Tn, 256)).astype(np.float32)
    V = rng.standard_normal((Tn, 256)).astype(np.float32)
    s = (q.astype(np.float64) @ K.T.astype(np.float64)) / 16.0
    p = np.exp(s - s.max(-1, keepdims=True))
    ref = (p / p.sum(-1, keepdims=True)) @ V.astype(np.float64)
    out = P.attention_split(q, K, V, n_slices, n_chunks)
    assert np.abs(out - ref).max() < 1e-10 * max(1.0, np.abs(ref).max())
