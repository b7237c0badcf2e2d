"""CPU oracle: numpy restatement of the reference's fp32 decode step.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import this module, and only as the
checker or the timed CPU baseline -- never as a product path.

It restates ``golden/model.py`` of allthingssecurity/qwen_fpga, the
reference's arithmetic contract, operation for operation in float32 numpy so
that it reproduces the golden's numbers (same op order, same dtypes, same
BLAS products).  Each method cites the lines it follows.  Parity of this port
is pinned against vectors that the unmodified reference golden produced in
the build container (``tests/golden/*.npz``, written by
``tests/golden/make_golden.py``).

Weights come from a packed blob (``qwen_fpga_b200.synth.Blob``); int8 tensors
are dequantised once (q * row scale, golden/quant.py:52-53) exactly like the
golden's fake-quant path.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

F32 = np.float32


def _sigm(x):
    # golden/model.py:54-55
    return 1.0 / (1.0 + np.exp(-x, dtype=F32))


def _silu(x):
    # golden/model.py:50-51
    return x / (1.0 + np.exp(-x, dtype=F32))


def _softplus(x):
    # golden/model.py:58-60: pass-through above 20
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def norm_1pw(x, w, eps):
    """(1+w)-gain RMSNorm over the last axis -- golden/model.py:63-75."""
    ms = np.mean(x.astype(F32) ** 2, axis=-1, keepdims=True)
    return (x * (1.0 / np.sqrt(ms + eps))) * (1.0 + w)


def unit_l2(x, eps=1e-6):
    """x / sqrt(sum x^2 + eps) over the last axis -- golden/model.py:78-80."""
    return x * (1.0 / np.sqrt(np.sum(x * x, axis=-1, keepdims=True) + eps))


def act_roundtrip(x, on):
    """Dynamic per-vector symmetric int8 fake-quant of an activation.

    golden/model.py:37-45 (the ACT_INT8 switch): s = amax/127 in float32,
    rint (half to even), clip to +-127, multiply back.  Identity when off or
    when the vector is all zero.
    """
    if not on:
        return x
    amax = np.abs(x).max()
    if amax == 0:
        return x
    s = amax / 127.0
    return np.rint(x / s).clip(-127, 127) * s


def act_int8(x):
    """The integer side of act_roundtrip: (q int8, s float32) with q*s the fake-quant.

    Same quantiser as scripts/export_gemv_tv.py:25-30 (scale 1.0 for an all-zero vector).
    """
    amax = np.abs(x).max()
    s = (amax / 127.0) if amax > 0 else F32(1.0)
    return np.rint(x / s).clip(-127, 127).astype(np.int8), F32(s)


def rope_table(pos, head_dim, partial, theta):
    """cos/sin of one position for the rotated slice -- golden/model.py:113-120."""
    rd = int(head_dim * partial)
    inv = 1.0 / (theta ** (np.arange(0, rd, 2, dtype=F32) / rd))
    ang = pos * inv
    ang2 = np.concatenate([ang, ang])
    return np.cos(ang2).astype(F32), np.sin(ang2).astype(F32)


def rotate(x, cos, sin):
    """Partial rotate-half RoPE on the first len(cos) dims -- golden/model.py:123-129."""
    rd = cos.shape[-1]
    h = rd // 2
    a, rest = x[..., :rd], x[..., rd:]
    rh = np.concatenate([-a[..., h:], a[..., :h]], axis=-1)
    return np.concatenate([a * cos + rh * sin, rest], axis=-1)


@dataclass
class PortState:
    """Recurrent decode state -- golden/model.py:86-107."""
    conv: np.ndarray                       # [n_linear, conv_dim, 4]
    rec: np.ndarray                        # [n_linear, H, K, V]
    kc: list = field(default_factory=list)  # per attention layer [T, nkv, hd]
    vc: list = field(default_factory=list)
    pos: int = 0

    @classmethod
    def zeros(cls, cfg):
        kinds = cfg["layer_types"]
        n_lin = kinds.count("linear_attention")
        n_full = kinds.count("full_attention")
        kd = cfg["linear_key_head_dim"] * cfg["linear_num_key_heads"]
        conv_dim = 2 * kd + cfg["linear_value_head_dim"] * cfg["linear_num_value_heads"]
        nkv, hd = cfg["num_key_value_heads"], cfg["head_dim"]
        return cls(
            conv=np.zeros((n_lin, conv_dim, cfg["linear_conv_kernel_dim"]), F32),
            rec=np.zeros((n_lin, cfg["linear_num_value_heads"], cfg["linear_key_head_dim"],
                          cfg["linear_value_head_dim"]), F32),
            kc=[np.zeros((0, nkv, hd), F32) for _ in range(n_full)],
            vc=[np.zeros((0, nkv, hd), F32) for _ in range(n_full)],
        )

    def copy(self):
        return PortState(self.conv.copy(), self.rec.copy(), [k.copy() for k in self.kc],
                         [v.copy() for v in self.vc], self.pos)


class PortDecoder:
    """One token in, logits out; mutates a PortState.  Mirrors golden decode_step."""

    def __init__(self, weights: dict, cfg: dict, act_int8: bool = False):
        self.W = weights
        self.cfg = cfg
        self.act_int8 = act_int8
        self.trace = None      # {"layer": i} -> filled like golden model.TRACE

    # ---------------------------------------------------------------- mixers
    def linear_mixer(self, pre, x, st, li):
        """Gated DeltaNet decode step -- golden/model.py:135-191."""
        c, W = self.cfg, self.W
        H, K, V = c["linear_num_value_heads"], c["linear_key_head_dim"], c["linear_value_head_dim"]
        kd = K * c["linear_num_key_heads"]
        eps = c["rms_norm_eps"]
        xa = act_roundtrip(x, self.act_int8)
        mixed = W[pre + "in_proj_qkv.weight"] @ xa           # :144
        z = W[pre + "in_proj_z.weight"] @ xa                 # :145
        b = W[pre + "in_proj_b.weight"] @ xa                 # :146
        a = W[pre + "in_proj_a.weight"] @ xa                 # :147
        # causal depthwise conv over [hist1..hist3, new], then SiLU (:149-155)
        taps = W[pre + "conv1d.weight"][:, 0, :]
        win = np.concatenate([st.conv[li], mixed[:, None]], axis=1)
        st.conv[li] = win[:, -4:]
        mixed = _silu(np.sum(win[:, 1:5] * taps, axis=1))
        q = mixed[:kd].reshape(H, K)
        k = mixed[kd:2 * kd].reshape(H, K)
        v = mixed[2 * kd:].reshape(H, V)
        beta = _sigm(b)                                                   # :161
        g = -np.exp(W[pre + "A_log"].astype(F32)) * _softplus(a + W[pre + "dt_bias"])  # :162
        q = unit_l2(q) * (K ** -0.5)                                      # :164
        k = unit_l2(k)                                                    # :165
        S = st.rec[li]
        tr = self.trace if (self.trace is not None and self.trace.get("layer") == li) else None
        if tr is not None:
            tr.update(q=q.copy(), k=k.copy(), v=v.copy(), g=g.copy(), beta=beta.copy(),
                      S_in=S.copy())
        # delta rule, in place (:174-178): decay, read k^T S, rank-1 write, read q^T S'
        S *= np.exp(g)[:, None, None]
        kS = np.einsum("hkv,hk->hv", S, k)
        d = (v - kS) * beta[:, None]
        S += np.einsum("hk,hv->hkv", k, d)
        o = np.einsum("hkv,hk->hv", S, q)
        if tr is not None:
            tr.update(o_core=o.copy(), S_out=S.copy())
        # gated RMSNorm: gain w (not 1+w), then * silu(z) (:183-189)
        zz = z.reshape(H, V)
        ms = np.mean(o.astype(F32) ** 2, axis=-1, keepdims=True)
        o = o * (1.0 / np.sqrt(ms + eps))
        o = W[pre + "norm.weight"] * o
        o = o * _silu(zz)
        return W[pre + "out_proj.weight"] @ act_roundtrip(o.reshape(-1), self.act_int8)  # :191

    def attn_mixer(self, pre, x, st, fi, pos):
        """Gated GQA full attention decode step -- golden/model.py:194-230."""
        c, W = self.cfg, self.W
        nh, nkv, hd = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
        eps = c["rms_norm_eps"]
        xa = act_roundtrip(x, self.act_int8)
        qg = (W[pre + "q_proj.weight"] @ xa).reshape(nh, 2 * hd)       # [q | gate] per head
        q, gate = qg[:, :hd], qg[:, hd:].reshape(-1)
        q = norm_1pw(q, W[pre + "q_norm.weight"], eps)
        k = norm_1pw((W[pre + "k_proj.weight"] @ xa).reshape(nkv, hd), W[pre + "k_norm.weight"], eps)
        v = (W[pre + "v_proj.weight"] @ xa).reshape(nkv, hd)
        rp = c["rope_parameters"]
        part = rp.get("partial_rotary_factor", c.get("partial_rotary_factor", 1.0))
        cos, sin = rope_table(pos, hd, part, rp["rope_theta"])
        q = rotate(q, cos, sin)
        k = rotate(k, cos, sin)
        st.kc[fi] = np.concatenate([st.kc[fi], k[None]], axis=0)       # roped K cached
        st.vc[fi] = np.concatenate([st.vc[fi], v[None]], axis=0)       # raw V cached
        rep = nh // nkv
        Kx = np.repeat(st.kc[fi], rep, axis=1)
        Vx = np.repeat(st.vc[fi], rep, axis=1)
        s = np.einsum("hd,thd->ht", q, Kx) * (hd ** -0.5)
        s = s - s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        o = np.einsum("ht,thd->hd", p, Vx).reshape(-1)
        o = o * _sigm(gate)
        return W[pre + "o_proj.weight"] @ act_roundtrip(o, self.act_int8)

    def ffn(self, pre, x):
        """SwiGLU MLP -- golden/model.py:233-237."""
        W = self.W
        xa = act_roundtrip(x, self.act_int8)
        g = _silu(W[pre + "gate_proj.weight"] @ xa)
        u = W[pre + "up_proj.weight"] @ xa
        return W[pre + "down_proj.weight"] @ act_roundtrip(g * u, self.act_int8)

    # ---------------------------------------------------------------- step
    def hidden(self, tok, st):
        """Embed + 24 layers, before the final norm -- golden/model.py:243-263."""
        c, W = self.cfg, self.W
        eps = c["rms_norm_eps"]
        h = W["embed_tokens.weight"][tok].copy()
        li = fi = 0
        for i, kind in enumerate(c["layer_types"]):
            pre = f"layers.{i}."
            res = h
            h = norm_1pw(h, W[pre + "input_layernorm.weight"], eps)
            if kind == "linear_attention":
                h = self.linear_mixer(pre + "linear_attn.", h, st, li)
                li += 1
            else:
                h = self.attn_mixer(pre + "self_attn.", h, st, fi, st.pos)
                fi += 1
            h = res + h
            res = h
            h = norm_1pw(h, W[pre + "post_attention_layernorm.weight"], eps)
            h = res + self.ffn(pre + "mlp.", h)
        return h

    def step(self, tok, st):
        """golden/model.py:243-267: returns fp32 logits [vocab] and advances st.pos."""
        h = self.hidden(tok, st)
        st.pos += 1
        h = norm_1pw(h, self.W["norm.weight"], self.cfg["rms_norm_eps"])
        return self.W["embed_tokens.weight"] @ h

    def greedy(self, prompt, n_new, st=None):
        """Prefill one token at a time, then greedy decode (golden/model.py:270-280).

        Returns (generated ids, per-step argmax of every call, final state).
        """
        st = st if st is not None else PortState.zeros(self.cfg)
        logits = None
        argmaxes = []
        for t in prompt:
            logits = self.step(int(t), st)
            argmaxes.append(int(np.argmax(logits)))
        out = []
        for _ in range(n_new):
            nxt = int(np.argmax(logits))
            out.append(nxt)
            logits = self.step(nxt, st)
            argmaxes.append(int(np.argmax(logits)))
        return out, argmaxes, st


def delta_rule_steps(S, q, k, v, g, beta):
    """The golden's recurrence (golden/model.py:174-178) over n tokens of one
    head: S [K, V]; q, k [n, K]; v [n, V]; g, beta [n].  Returns (o [n, V],
    S after the n tokens); float32, S not modified."""
    S = S.astype(F32).copy()
    o = np.empty((len(g), S.shape[1]), F32)
    for t in range(len(g)):
        S *= np.exp(F32(g[t]))
        d = (v[t] - k[t] @ S) * F32(beta[t])
        S += np.outer(k[t], d).astype(F32)
        o[t] = q[t] @ S
    return o, S


def delta_rule_chunk(S, q, k, v, g, beta):
    """The same n tokens in the chunked (WY) form the GPU prefill computes.
    With G_t = g_0 + ... + g_t and Gamma_t = e^{G_t}:
      d_t = beta_t (v_t - Gamma_t S^T k_t) - sum_{s<t} beta_t e^{G_t-G_s} (k_t.k_s) d_s
      o_t = Gamma_t S^T q_t + sum_{s<=t} e^{G_t-G_s} (q_t.k_s) d_s
      S'  = Gamma_{n-1} S + sum_t e^{G_{n-1}-G_t} k_t d_t^T
    (one triangular solve for d, then dense products).  float32."""
    n = len(g)
    G = np.cumsum(np.asarray(g, F32)).astype(F32)
    dec = np.exp(G[:, None] - G[None, :]).astype(F32)          # e^{G_t - G_s}
    low = np.tril(np.ones((n, n), bool), -1)
    A = np.where(low, beta[:, None] * dec * (k @ k.T), 0).astype(F32)
    R = (beta[:, None] * (v - np.exp(G)[:, None] * (k @ S))).astype(F32)
    D = np.zeros_like(R)
    for t in range(n):                                         # (I + A) D = R, forward substitution
        D[t] = R[t] - A[t, :t] @ D[:t]
    QK = np.where(np.tril(np.ones((n, n), bool)), dec * (q @ k.T), 0).astype(F32)
    o = (np.exp(G)[:, None] * (q @ S) + QK @ D).astype(F32)
    w = np.exp(G[-1] - G).astype(F32)
    S2 = (np.exp(G[-1]) * S + (k * w[:, None]).T @ D).astype(F32)
    return o, S2


def attention_split(q, K, V, n_slices, n_chunks):
    """The decomposition the decode kernel uses for golden/model.py:219-229
    (softmax(q K^T / sqrt(hd)) V for one KV group's query heads): the Tn
    positions cut into n_slices rank slices [j Tn / n, (j + 1) Tn / n), each
    cut into at most n_chunks chunks of ceil(len / chunks) positions; per chunk
    (m, l, o) = (max score, sum of exp(s - m), sum of exp(s - m) v); chunks and
    then slices combined in order, empty ones (m = -inf) skipped.
    q [H, hd], K / V [Tn, hd]; returns [H, hd]."""
    q, K, V = (np.asarray(a, np.float64) for a in (q, K, V))
    Tn, hd = K.shape
    scale = hd ** -0.5

    def part(t0, t1):
        if t1 <= t0:
            return (np.full(q.shape[0], -np.inf), np.zeros(q.shape[0]), np.zeros_like(q))
        s = (q @ K[t0:t1].T) * scale
        m = s.max(-1)
        e = np.exp(s - m[:, None])
        return m, e.sum(-1), e @ V[t0:t1]

    def merge(parts):
        M, L, O = np.full(q.shape[0], -np.inf), np.zeros(q.shape[0]), np.zeros_like(q)
        for m, l, o in parts:
            if np.all(m == -np.inf):
                continue
            Mn = np.maximum(M, m)
            a = np.where(M == -np.inf, 0.0, np.exp(M - Mn))
            b = np.exp(m - Mn)
            L, O, M = L * a + l * b, O * a[:, None] + o * b[:, None], Mn
        return M, L, O

    slices = []
    for j in range(n_slices):
        s0, s1 = j * Tn // n_slices, (j + 1) * Tn // n_slices
        n = max(1, min(n_chunks, -(-(s1 - s0) // 16)))
        cl = -(-(s1 - s0) // n)
        slices.append(merge([part(s0 + c * cl, min(s1, s0 + c * cl + cl)) for c in range(n)]))
    M, L, O = merge(slices)
    return O / L[:, None]


def gemv_int32(w_i8: np.ndarray, x_i8: np.ndarray) -> np.ndarray:
    """Exact int32 accumulators acc[o] = sum_i w[o,i]*x[i] (scripts/export_gemv_tv.py:49)."""
    return (w_i8.astype(np.int32) @ x_i8.astype(np.int32)).astype(np.int32)


def gemv_dequant(acc: np.ndarray, sx, sw: np.ndarray) -> np.ndarray:
    """acc * sx * sw in float32, the dequant of scripts/export_gemv_tv.py:50."""
    return acc.astype(F32) * F32(sx) * sw


def warm_state(cfg, T, seed=2, rec_std=0.1, kv_std=1.0):
    """Warm start of the W8A8 / long-context configs: DeltaNet states N(0, rec_std),
    conv history zero, T cached positions of K (post-RoPE) and V drawn N(0, kv_std),
    pos = T.  Drawn from default_rng(seed) in the order rec, then per attention
    layer K then V."""
    st = PortState.zeros(cfg)
    rng = np.random.default_rng(seed)
    st.rec[...] = rng.standard_normal(st.rec.shape, F32) * F32(rec_std)
    nkv, hd = cfg["num_key_value_heads"], cfg["head_dim"]
    for f in range(len(st.kc)):
        st.kc[f] = rng.standard_normal((T, nkv, hd), F32) * F32(kv_std)
        st.vc[f] = rng.standard_normal((T, nkv, hd), F32) * F32(kv_std)
    st.pos = T
    return st
