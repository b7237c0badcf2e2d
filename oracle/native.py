"""ctypes loaders for the compiled CPU checkers in oracle/ (test infrastructure only).

* ``HlsRef``   -- the reference's own HLS C++ decoder (``_ref/libqwen_hls_ref.so``,
  built by ``make -C oracle ref`` from the reference checkout).  Runs qwen_top
  (hls/src/qwen_synth.hpp:39-92) on the packed blob, single thread.
* ``gemv_i8_i8`` / ``gemv_i8_f32`` -- the C restatement in gemv_port.c.
"""

from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB = os.path.join(HERE, "_ref", "libqwen_hls_ref.so")
PORT_LIB = os.path.join(HERE, "_port", "libgemv_port.so")

_fp = C.POINTER(C.c_float)
_i8p = C.POINTER(C.c_int8)
_i32p = C.POINTER(C.c_int32)


def _p(a, t):
    return a.ctypes.data_as(t) if a is not None else None


def reference_checkout() -> str | None:
    """The reference checkout: $QWEN_REF, else the reference_path that
    BASELINE.json at the repository root records (None if neither exists)."""
    ref = os.environ.get("QWEN_REF")
    if not ref:
        import json
        bj = os.path.join(os.path.dirname(HERE), "BASELINE.json")
        if os.path.exists(bj):
            with open(bj) as f:
                ref = json.load(f).get("reference_path")
    return ref if ref and os.path.isdir(ref) else None


def build(ref: str | None = None) -> None:
    """Compile the C port, and the reference shim when the reference checkout exists."""
    import subprocess
    subprocess.run(["make", "-s", "-C", HERE, "port"], check=True)
    ref = ref or reference_checkout()
    if ref and os.path.isdir(os.path.join(ref, "hls", "src")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref}"], check=True)


def have_ref() -> bool:
    return os.path.exists(REF_LIB)


class HlsRef:
    """One reference DecodeState driven through qwen_top."""

    MAX_CTX = 8192

    def __init__(self, blob_path: str):
        if not have_ref():
            raise FileNotFoundError(f"{REF_LIB} missing: run `make -C oracle ref`")
        self.lib = C.CDLL(REF_LIB)
        L = self.lib
        L.hls_ref_new.restype = C.c_void_p
        L.hls_ref_free.argtypes = [C.c_void_p]
        L.hls_ref_reset.argtypes = [C.c_void_p]
        L.hls_ref_set_state.argtypes = [C.c_void_p, _fp, _fp, _fp, _fp, C.c_int, C.c_int]
        L.hls_ref_step.argtypes = [C.c_void_p, C.c_void_p, C.c_int, _fp]
        L.hls_ref_pos.argtypes = [C.c_void_p]
        L.hls_ref_delta_rule_layer.argtypes = [_fp] * 7
        L.hls_ref_gemv_i8.argtypes = [_fp, _i8p, _fp, _fp, C.c_int, C.c_int]
        self.blob = np.fromfile(blob_path, dtype=np.uint8)
        self.st = L.hls_ref_new()

    def close(self):
        if self.st:
            self.lib.hls_ref_free(self.st)
            self.st = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        self.lib.hls_ref_reset(self.st)

    def set_state(self, conv, rec, kc, vc, pos):
        """kc/vc: [6, T, 2, 256] float32 (post-RoPE K, raw V)."""
        conv = np.ascontiguousarray(conv, np.float32)
        rec = np.ascontiguousarray(rec, np.float32)
        kc = np.ascontiguousarray(kc, np.float32)
        vc = np.ascontiguousarray(vc, np.float32)
        T = kc.shape[1]
        if T != pos:
            raise ValueError("qwen_top appends at slot pos, so the cache length must equal pos")
        rc = self.lib.hls_ref_set_state(self.st, _p(conv, _fp), _p(rec, _fp), _p(kc, _fp),
                                        _p(vc, _fp), T, pos)
        if rc != 0:
            raise ValueError("state rejected (context beyond the HLS 8192 limit?)")

    def step(self, tok: int, want_logits: bool = False):
        lg = np.empty(248320, np.float32) if want_logits else None
        am = self.lib.hls_ref_step(self.blob.ctypes.data_as(C.c_void_p), self.st, int(tok),
                                   _p(lg, _fp))
        if am < 0:
            raise ValueError("context beyond the HLS 8192 limit")
        return am, lg

    def delta_rule_layer(self, q, k, v, g, beta, S):
        S = np.array(S, np.float32, copy=True, order="C")
        out = np.empty((16, 128), np.float32)
        args = [np.ascontiguousarray(a, np.float32) for a in (q, k, v, g, beta)]
        self.lib.hls_ref_delta_rule_layer(*[_p(a, _fp) for a in args], _p(S, _fp), _p(out, _fp))
        return out, S


_port = None


def _port_lib():
    global _port
    if _port is None:
        if not os.path.exists(PORT_LIB):
            raise FileNotFoundError(f"{PORT_LIB} missing: run `make -C oracle port`")
        L = C.CDLL(PORT_LIB)
        L.gemv_port_i8_i8.argtypes = [_i32p, _fp, _i8p, _fp, _i8p, C.c_float, C.c_long,
                                      C.c_long, C.c_int]
        L.gemv_port_i8_f32.argtypes = [_fp, _i8p, _fp, _fp, C.c_long, C.c_long, C.c_int]
        _port = L
    return _port


def gemv_i8_i8(w, sw, x, sx, threads=None):
    threads = threads or os.cpu_count() or 1
    n, k = w.shape
    acc = np.empty(n, np.int32)
    y = np.empty(n, np.float32)
    _port_lib().gemv_port_i8_i8(_p(acc, _i32p), _p(y, _fp), _p(np.ascontiguousarray(w), _i8p),
                                _p(np.ascontiguousarray(sw, np.float32), _fp),
                                _p(np.ascontiguousarray(x), _i8p), float(sx), n, k, threads)
    return acc, y


def gemv_i8_f32(w, s, x, threads=None):
    threads = threads or os.cpu_count() or 1
    n, k = w.shape
    y = np.empty(n, np.float32)
    _port_lib().gemv_port_i8_f32(_p(y, _fp), _p(np.ascontiguousarray(w), _i8p),
                                 _p(np.ascontiguousarray(s, np.float32), _fp),
                                 _p(np.ascontiguousarray(x, np.float32), _fp), n, k, threads)
    return y
