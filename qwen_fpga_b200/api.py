"""ctypes binding of libqwenb200.so -- the Python face of the C ABI in
include/qwen_b200.h.

It mirrors the reference's decode interface so callers of
``golden/model.py`` can switch with a one-line change:

    golden                                       this package
    -------------------------------------------  -----------------------------------------
    DecodeState.new(cfg)       (model.py:97)     Decoder(blob).state()  /  dec.reset()
    decode_step(W, cfg, tok, st) (model.py:243)  decode_step(dec, cfg, tok, st)
    generate(W, cfg, ids, n)   (model.py:270)    generate(dec, cfg, ids, n)
    model.ACT_INT8 = True      (model.py:34)     dec.set_act_int8(True)

There is no CPU fallback: if the library is missing or no CUDA device is
present the calls raise.
"""

from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqwenb200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "qwen_b200.h")
VOCAB = 248320

QWEN_OK, QWEN_ERR_ARG, QWEN_ERR_IO, QWEN_ERR_CUDA, QWEN_ERR_DEVICE, QWEN_ERR_STATE = range(6)

_fp = C.POINTER(C.c_float)
_ip = C.POINTER(C.c_int)
_i8p = C.POINTER(C.c_int8)
_i32p = C.POINTER(C.c_int32)
_vp = C.c_void_p

_lib = None


class QwenError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"qwen error {code}: {msg}")
        self.code = code


def header_symbols() -> list[str]:
    """Function names declared in include/qwen_b200.h."""
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(qwen_\w+)\s*\(", txt, re.M)))


def load() -> C.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(f"{LIB_PATH} missing: run `python -m qwen_fpga_b200.build`")
    L = C.CDLL(LIB_PATH)
    L.qwen_version.restype = C.c_char_p
    L.qwen_last_error.restype = C.c_char_p
    L.qwen_last_error.argtypes = [_vp]
    L.qwen_create.argtypes = [C.c_char_p, C.c_char_p, C.c_int, _ip, C.c_int, C.c_int,
                              C.POINTER(_vp)]
    L.qwen_create_tp.argtypes = [C.c_char_p, C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                 C.POINTER(_vp)]
    L.qwen_tp_export.argtypes = [_vp, _vp]
    L.qwen_tp_connect.argtypes = [_vp, _vp]
    L.qwen_tp_vocab_range.argtypes = [_vp, _ip, _ip]
    L.qwen_tp_plan.argtypes = [C.c_int, C.c_int, _ip]
    L.qwen_pack_blob.argtypes = [C.c_char_p, C.c_char_p]
    L.qwen_destroy.argtypes = [_vp]
    L.qwen_reset.argtypes = [_vp, C.c_int]
    L.qwen_state_import.argtypes = [_vp, C.c_int, _fp, _fp, _fp, _fp, C.c_int, C.c_int]
    L.qwen_state_export.argtypes = [_vp, C.c_int, _fp, _fp, _fp, _fp, _ip, _ip]
    L.qwen_set_act_int8.argtypes = [_vp, C.c_int]
    L.qwen_trace_enable.argtypes = [_vp, C.c_int]
    L.qwen_trace_read.argtypes = [_vp, C.POINTER(C.c_ulonglong), C.c_int, _ip, _ip]
    L.qwen_decode_step.argtypes = [_vp, _ip, C.c_int, _vp, _ip]
    L.qwen_generate.argtypes = [_vp, _ip, C.c_int, C.c_int, _ip, C.POINTER(C.c_double)]
    L.qwen_gemv_i8_f32.argtypes = [_vp, _vp, _vp, _vp, C.c_int, C.c_int, _vp]
    L.qwen_gemv_i8_i8.argtypes = [_vp, _vp, _vp, _vp, _vp, C.c_float, C.c_int, C.c_int, _vp]
    L.qwen_gemm_i8_i8.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp]
    L.qwen_decode_timed.argtypes = [_vp, C.c_int, C.c_int, C.POINTER(C.c_double)]
    L.qwen_prefill.argtypes = [_vp, _ip, C.c_int, _vp, _ip]
    L.qwen_delta_rule_layer.argtypes = [_vp] * 7 + [_vp]
    L.qwen_gemv_i8_f32_argmax_noalloc.argtypes = [_vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int, _vp]
    L.qwen_capture_phase.argtypes = [_vp, C.c_int]
    L.qwen_capture_read.argtypes = [_vp, _fp, C.c_int]
    _lib = L
    return L


def _check(rc, ctx=None):
    if rc != QWEN_OK:
        msg = load().qwen_last_error(ctx).decode(errors="replace")
        raise QwenError(rc, msg)


def _fptr(a):
    return a.ctypes.data_as(_fp) if a is not None else None


TP_HANDLE_BYTES = 64


def pack_blob(snapshot_dir: str, out_blob: str) -> str:
    """Pack a safetensors snapshot of the Qwen3.5 text decoder into the blob
    Decoder loads (scripts/pack_weights.py's layout, in C++; host only).
    Writes out_blob, <stem>.manifest.json and <stem>.idx; returns the index path."""
    _check(load().qwen_pack_blob(snapshot_dir.encode(), out_blob.encode()))
    return os.path.splitext(out_blob)[0] + ".idx"


def tp_plan(rank: int, world: int) -> dict:
    """The tensor-parallel shard of `rank` among `world` GPUs (no GPU needed):
    DeltaNet heads, attention KV groups, OUT input columns, FFN columns and
    vocab rows, each as a half-open [lo, hi) pair."""
    out = (C.c_int * 10)()
    _check(load().qwen_tp_plan(int(rank), int(world), out))
    v = list(out)
    return {"dn_heads": (v[0], v[1]), "kv_groups": (v[2], v[3]), "out_cols": (v[4], v[5]),
            "ffn_cols": (v[6], v[7]), "vocab": (v[8], v[9])}


class DecodeStateView:
    """Host copy of the decode state, field for field the golden DecodeState
    (golden/model.py:86-95): conv [18,6144,4], rec [18,16,128,128], kc/vc lists
    of [T,2,256] per attention layer, pos."""

    def __init__(self, conv, rec, kc, vc, pos):
        self.conv, self.rec, self.kc, self.vc, self.pos = conv, rec, kc, vc, pos


class Decoder:
    """One GPU context: weights resident in HBM + one batch-1 decode state."""

    def __init__(self, blob_path: str, index_path: str | None = None, device: int = 0,
                 max_ctx: int = 4096, act_int8: bool = False, tp_rank: int = 0, tp_world: int = 1):
        """tp_world > 1: rank tp_rank of a tensor-parallel job (one Decoder per
        GPU and process); connect the ranks with tp_handle / tp_connect before
        decoding (qwen_fpga_b200.tp does it over torch.distributed)."""
        L = load()
        if index_path is None:
            index_path = os.path.splitext(blob_path)[0] + ".idx"
        self.max_ctx = max_ctx
        self.tp_rank, self.tp_world = int(tp_rank), int(tp_world)
        h = _vp()
        if self.tp_world == 1:
            dev = (C.c_int * 1)(device)
            rc = L.qwen_create(blob_path.encode(), index_path.encode(), 1, dev, max_ctx, 1,
                               C.byref(h))
        else:
            rc = L.qwen_create_tp(blob_path.encode(), index_path.encode(), int(device), self.tp_rank,
                                  self.tp_world, max_ctx, 1, C.byref(h))
        _check(rc)
        self.h = h
        self.act_int8 = False
        if act_int8:
            self.set_act_int8(True)

    def close(self):
        if getattr(self, "h", None):
            load().qwen_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def tp_handle(self) -> bytes:
        """This rank's exchange-buffer handle (TP_HANDLE_BYTES bytes)."""
        buf = C.create_string_buffer(TP_HANDLE_BYTES)
        _check(load().qwen_tp_export(self.h, buf), self.h)
        return buf.raw

    def tp_connect(self, handles):
        """handles: every rank's tp_handle() in rank order."""
        if len(handles) != self.tp_world or any(len(x) != TP_HANDLE_BYTES for x in handles):
            raise ValueError("need tp_world handles of TP_HANDLE_BYTES bytes")
        buf = C.create_string_buffer(b"".join(handles), TP_HANDLE_BYTES * self.tp_world)
        _check(load().qwen_tp_connect(self.h, buf), self.h)

    @property
    def vocab_range(self) -> tuple[int, int]:
        """Rows of the logits this context fills: all of them, or the rank's vocab slice."""
        lo, hi = C.c_int(), C.c_int()
        _check(load().qwen_tp_vocab_range(self.h, C.byref(lo), C.byref(hi)), self.h)
        return lo.value, hi.value

    def set_act_int8(self, on: bool):
        _check(load().qwen_set_act_int8(self.h, 1 if on else 0), self.h)
        self.act_int8 = bool(on)

    def trace_enable(self, on: bool = True):
        _check(load().qwen_trace_enable(self.h, 1 if on else 0), self.h)

    def trace_read(self):
        """Last step's per-CTA, per-phase stamps [entry, inputs arrived, outputs written, exit] (ns),
        shape [n_ctas, n_phases, 4]; CTA 0's per-warp clock stamps land in
        self.trace_warps, shape [n_phases, 16, 16]."""
        n = 160 * 121 * 4 + 121 * 16 * 16
        buf = np.zeros(n, np.uint64)
        nc, npz = C.c_int(), C.c_int()
        _check(load().qwen_trace_read(self.h, buf.ctypes.data_as(C.POINTER(C.c_ulonglong)), n,
                                      C.byref(nc), C.byref(npz)), self.h)
        m = nc.value * npz.value * 4
        self.trace_warps = buf[m:m + npz.value * 16 * 16].reshape(npz.value, 16, 16)
        return buf[:m].reshape(nc.value, npz.value, 4)

    def reset(self):
        _check(load().qwen_reset(self.h, 0), self.h)

    CAPTURE_FLOATS = 16392

    def capture_phase(self, phase: int):
        """Arm (phase >= 0) or disarm (-1) the W8A8 capture of one GEMV phase."""
        _check(load().qwen_capture_phase(self.h, int(phase)), self.h)

    def capture_read(self) -> dict:
        """The last armed step's capture: x (fp32 input), xq (int8), sx, K, acc (int32 rows)."""
        buf = np.zeros(self.CAPTURE_FLOATS, np.float32)
        _check(load().qwen_capture_read(self.h, buf.ctypes.data_as(_fp), buf.size), self.h)
        K = int(buf[8193])
        return {"captured": bool(buf[8194] != 0), "K": K, "x": buf[:K].copy(),
                "xq": buf[4096:4096 + K].astype(np.int8), "sx": np.float32(buf[8192]),
                "acc": buf[8200:].view(np.int32).copy()}

    def decode_step(self, tok: int, want_logits: bool = True, out=None):
        """Returns (argmax, logits or None).  `out` (optional): a float32 array of
        VOCAB elements the logits are written into (e.g. pinned host memory);
        it is returned as the logits."""
        t = (C.c_int * 1)(int(tok))
        am = (C.c_int * 1)()
        if out is not None:
            if out.dtype != np.float32 or out.size != VOCAB or not out.flags["C_CONTIGUOUS"]:
                raise ValueError("out must be a contiguous float32 array of VOCAB elements")
            lg = out
        else:
            lg = np.empty(VOCAB, np.float32) if want_logits else None
        rc = load().qwen_decode_step(self.h, t, 1, lg.ctypes.data if lg is not None else None, am)
        _check(rc, self.h)
        return int(am[0]), lg

    def prefill(self, tokens, want_logits: bool = True):
        """All prompt tokens through the layers at once (qwen_prefill): the
        state afterwards is that of one decode_step per token.  Returns the
        last token's (argmax, logits or None)."""
        t = np.ascontiguousarray(np.asarray(tokens, np.int32))
        am = (C.c_int * 1)()
        lg = np.empty(VOCAB, np.float32) if want_logits else None
        _check(load().qwen_prefill(self.h, t.ctypes.data_as(_ip), int(t.size),
                                   lg.ctypes.data if lg is not None else None, am), self.h)
        return int(am[0]), lg

    def generate(self, prompt, n_new: int):
        """Prefill + greedy decode; returns (ids, decode seconds)."""
        p = np.ascontiguousarray(np.asarray(prompt, np.int32))
        out = np.empty(max(n_new, 1), np.int32)
        sec = C.c_double()
        rc = load().qwen_generate(self.h, p.ctypes.data_as(_ip), len(p), int(n_new),
                                  out.ctypes.data_as(_ip), C.byref(sec))
        _check(rc, self.h)
        return [int(v) for v in out[:n_new]], sec.value

    def import_state(self, st):
        """st: golden DecodeState or anything with conv/rec/kc/vc/pos (kc/vc per layer [T,2,256])."""
        conv = np.ascontiguousarray(st.conv, np.float32)
        rec = np.ascontiguousarray(st.rec, np.float32)
        T = int(st.kc[0].shape[0]) if len(st.kc) else 0
        if T:
            kc = np.ascontiguousarray(np.stack([np.asarray(k, np.float32) for k in st.kc]))
            vc = np.ascontiguousarray(np.stack([np.asarray(v, np.float32) for v in st.vc]))
        else:
            kc = vc = None
        rc = load().qwen_state_import(self.h, 0, _fptr(conv), _fptr(rec), _fptr(kc), _fptr(vc),
                                      T, int(st.pos))
        _check(rc, self.h)

    def export_state(self) -> DecodeStateView:
        T = C.c_int()
        pos = C.c_int()
        L = load()
        _check(L.qwen_state_export(self.h, 0, None, None, None, None, C.byref(T), C.byref(pos)),
               self.h)
        conv = np.empty((18, 6144, 4), np.float32)
        rec = np.empty((18, 16, 128, 128), np.float32)
        kc = np.empty((6, T.value, 2, 256), np.float32)
        vc = np.empty((6, T.value, 2, 256), np.float32)
        rc = L.qwen_state_export(self.h, 0, _fptr(conv), _fptr(rec),
                                 _fptr(kc) if T.value else None, _fptr(vc) if T.value else None,
                                 C.byref(T), C.byref(pos))
        _check(rc, self.h)
        return DecodeStateView(conv, rec, list(kc), list(vc), pos.value)


class BatchDecoder:
    """One GPU context holding max_batch sequences, each with its own decode
    state (golden/model.py:86-107), stepped together (golden/model.py:243-267
    per sequence) by the batched engine: int8 projections on tcgen05 over the
    batch's tokens."""

    def __init__(self, blob_path: str, max_batch: int, index_path: str | None = None, device: int = 0,
                 max_ctx: int = 4096, act_int8: bool = True):
        L = load()
        if index_path is None:
            index_path = os.path.splitext(blob_path)[0] + ".idx"
        self.max_ctx, self.max_batch = int(max_ctx), int(max_batch)
        h = _vp()
        dev = (C.c_int * 1)(device)
        _check(L.qwen_create(blob_path.encode(), index_path.encode(), 1, dev, self.max_ctx, self.max_batch,
                             C.byref(h)))
        self.h = h
        self.set_act_int8(act_int8)

    def close(self):
        if getattr(self, "h", None):
            load().qwen_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_act_int8(self, on: bool):
        _check(load().qwen_set_act_int8(self.h, 1 if on else 0), self.h)
        self.act_int8 = bool(on)

    def reset(self, seq: int = -1):
        """Zero sequence seq's state (-1: every sequence)."""
        _check(load().qwen_reset(self.h, int(seq)), self.h)

    def import_state(self, seq: int, st):
        """st: a golden DecodeState (conv, rec, kc / vc lists of [T,2,256], pos) for sequence seq."""
        conv = np.ascontiguousarray(st.conv, np.float32)
        rec = np.ascontiguousarray(st.rec, np.float32)
        T = int(st.kc[0].shape[0]) if len(st.kc) else 0
        kc = np.ascontiguousarray(np.stack([np.asarray(k, np.float32) for k in st.kc])) if T else None
        vc = np.ascontiguousarray(np.stack([np.asarray(v, np.float32) for v in st.vc])) if T else None
        _check(load().qwen_state_import(self.h, int(seq), _fptr(conv), _fptr(rec), _fptr(kc), _fptr(vc), T,
                                        int(st.pos)), self.h)

    def export_state(self, seq: int) -> DecodeStateView:
        T, pos = C.c_int(), C.c_int()
        L = load()
        _check(L.qwen_state_export(self.h, int(seq), None, None, None, None, C.byref(T), C.byref(pos)), self.h)
        conv = np.empty((18, 6144, 4), np.float32)
        rec = np.empty((18, 16, 128, 128), np.float32)
        kc = np.empty((6, T.value, 2, 256), np.float32)
        vc = np.empty((6, T.value, 2, 256), np.float32)
        _check(L.qwen_state_export(self.h, int(seq), _fptr(conv), _fptr(rec), _fptr(kc) if T.value else None,
                                   _fptr(vc) if T.value else None, C.byref(T), C.byref(pos)), self.h)
        return DecodeStateView(conv, rec, list(kc), list(vc), pos.value)

    def step(self, toks, want_logits: bool = False, out=None):
        """One step of sequences 0 .. len(toks)-1, toks[b] feeding sequence b.
        Returns (argmax list, logits [B, VOCAB] or None); `out` (optional): a
        float32 array of B * VOCAB elements the logits are written into."""
        t = np.ascontiguousarray(np.asarray(toks, np.int32))
        B = int(t.size)
        am = np.empty(B, np.int32)
        lg = None
        if out is not None:
            if out.dtype != np.float32 or out.size != B * VOCAB or not out.flags["C_CONTIGUOUS"]:
                raise ValueError("out must be a contiguous float32 array of B * VOCAB elements")
            lg = out
        elif want_logits:
            lg = np.empty((B, VOCAB), np.float32)
        _check(load().qwen_decode_step(self.h, t.ctypes.data_as(_ip), B, lg.ctypes.data if lg is not None else None,
                                       am.ctypes.data_as(_ip)), self.h)
        return [int(v) for v in am], lg

    def step_greedy(self, batch: int, want_logits: bool = False):
        """One step in which every sequence b < batch takes its previous argmax."""
        am = np.empty(batch, np.int32)
        lg = np.empty((batch, VOCAB), np.float32) if want_logits else None
        _check(load().qwen_decode_step(self.h, None, int(batch), lg.ctypes.data if lg is not None else None,
                                       am.ctypes.data_as(_ip)), self.h)
        return [int(v) for v in am], lg

    def timed(self, batch: int, steps: int) -> float:
        """`steps` greedy steps of sequences 0 .. batch-1; device seconds."""
        sec = C.c_double()
        _check(load().qwen_decode_timed(self.h, int(batch), int(steps), C.byref(sec)), self.h)
        return sec.value


# ---------------------------------------------------------------- golden-shaped façade

def decode_step(dec: Decoder, cfg, tok: int, st=None):
    """Drop-in for golden/model.py:243 decode_step: returns fp32 logits [vocab].

    The state lives on the GPU inside ``dec``; ``st`` is accepted for signature
    compatibility and, if it carries a ``pos`` attribute, advanced like the
    golden's ``st.pos += 1``."""
    _, lg = dec.decode_step(tok, want_logits=True)
    if st is not None and hasattr(st, "pos"):
        st.pos += 1
    return lg


def generate(dec: Decoder, cfg, prompt_ids, n_new=16, greedy=True):
    """Drop-in for golden/model.py:270 generate (greedy only): returns (ids, None)."""
    ids, _ = dec.generate(prompt_ids, n_new)
    return ids, None


# ---------------------------------------------------------------- operators on torch tensors

def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _stream(stream):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _need(name, t, dtype, shape, device):
    """t must be a contiguous CUDA tensor of `dtype` and `shape` on `device`."""
    if t is None:
        raise ValueError(f"{name} is required")
    if not t.is_cuda or t.device != device:
        raise ValueError(f"{name} must be a CUDA tensor on {device} (got {t.device})")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype} (got {t.dtype})")
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)} (got {tuple(t.shape)})")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _gemv_shape(w):
    import torch
    if w is None or w.dim() != 2:
        raise ValueError("w must be a 2-D [N, K] tensor")
    _need("w", w, torch.int8, tuple(w.shape), w.device)
    return w.shape


def gemv_i8_f32(w, s, x, y=None, stream=None):
    """y = s * (w @ x) for torch CUDA tensors w int8 [N,K], s fp32 [N], x fp32 [K]."""
    import torch
    N, K = _gemv_shape(w)
    y = y if y is not None else torch.empty(N, dtype=torch.float32, device=w.device)
    _need("s", s, torch.float32, (N,), w.device)
    _need("x", x, torch.float32, (K,), w.device)
    _need("y", y, torch.float32, (N,), w.device)
    with torch.cuda.device(w.device):
        rc = load().qwen_gemv_i8_f32(_ptr(y), _ptr(w), _ptr(s), _ptr(x), N, K, _stream(stream))
    _check(rc)
    return y


def gemv_i8_i8(w, sw, xq, sx, acc=None, y=None, stream=None, want_acc=True, want_y=True):
    """acc = w @ xq (int32, exact), y = acc * sx * sw for torch CUDA tensors."""
    import torch
    N, K = _gemv_shape(w)
    if want_acc and acc is None:
        acc = torch.empty(N, dtype=torch.int32, device=w.device)
    if want_y and y is None:
        y = torch.empty(N, dtype=torch.float32, device=w.device)
    _need("xq", xq, torch.int8, (K,), w.device)
    if want_acc:
        _need("acc", acc, torch.int32, (N,), w.device)
    if want_y:
        _need("y", y, torch.float32, (N,), w.device)
        _need("sw", sw, torch.float32, (N,), w.device)
    with torch.cuda.device(w.device):
        rc = load().qwen_gemv_i8_i8(_ptr(acc if want_acc else None), _ptr(y if want_y else None),
                                    _ptr(w), _ptr(sw), _ptr(xq), float(sx), N, K, _stream(stream))
    _check(rc)
    return acc, y


def gemm_i8_i8(w, sw, xq, sx, acc=None, y=None, stream=None, want_acc=True, want_y=True):
    """Batched int8 x int8 projection on the tensor cores: acc[b] = w @ xq[b]
    (int32, exact), y[b] = acc[b] * sx[b] * sw, for torch CUDA tensors w int8
    [N, K], sw fp32 [N], xq int8 [B, K], sx fp32 [B].  Returns (acc [B, N], y [B, N])."""
    import torch
    N, K = _gemv_shape(w)
    if xq is None or xq.dim() != 2:
        raise ValueError("xq must be a 2-D [B, K] tensor")
    B = int(xq.shape[0])
    _need("xq", xq, torch.int8, (B, K), w.device)
    _need("sx", sx, torch.float32, (B,), w.device)
    _need("sw", sw, torch.float32, (N,), w.device)
    if want_acc and acc is None:
        acc = torch.empty((B, N), dtype=torch.int32, device=w.device)
    if want_y and y is None:
        y = torch.empty((B, N), dtype=torch.float32, device=w.device)
    if want_acc:
        _need("acc", acc, torch.int32, (B, N), w.device)
    if want_y:
        _need("y", y, torch.float32, (B, N), w.device)
    with torch.cuda.device(w.device):
        rc = load().qwen_gemm_i8_i8(_ptr(acc if want_acc else None), _ptr(y if want_y else None), _ptr(w),
                                    _ptr(sw), _ptr(xq), _ptr(sx), N, K, B, _stream(stream))
    _check(rc)
    return acc, y


def gemv_i8_f32_argmax_noalloc(w, s, x, argmax, y=None, stream=None):
    """y = s * (w @ x) (when y is given) and argmax[0] = first index of its maximum,
    through the allocation-free entry point; argmax is a caller-owned int32 CUDA
    tensor of one element, y an optional fp32 [N] CUDA tensor.  Every tensor must
    be contiguous and on w's device; the call runs with that device current."""
    import torch
    N, K = _gemv_shape(w)
    _need("s", s, torch.float32, (N,), w.device)
    _need("x", x, torch.float32, (K,), w.device)
    _need("argmax", argmax, torch.int32, (1,), w.device)
    if y is not None:
        _need("y", y, torch.float32, (N,), w.device)
    with torch.cuda.device(w.device):
        rc = load().qwen_gemv_i8_f32_argmax_noalloc(_ptr(y), _ptr(argmax), _ptr(w), _ptr(s), _ptr(x), N,
                                                    K, _stream(stream))
    _check(rc)
    return y, argmax


def delta_rule_layer(q, k, v, g, beta, S, out=None, stream=None):
    """In-place gated delta rule of one 16-head layer on torch CUDA fp32 tensors."""
    import torch
    out = out if out is not None else torch.empty((16, 128), dtype=torch.float32, device=S.device)
    rc = load().qwen_delta_rule_layer(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(S),
                                      _ptr(out), _stream(stream))
    _check(rc)
    return out
