"""Synthetic Qwen3.5-0.8B weights written in the reference's packed-blob format.

There is no checkpoint on this machine, so every run uses a seeded random-init
model of the exact 0.8B shapes.  The blob is the reference's on-disk contract
(qwen_fpga ``scripts/pack_weights.py:1-101``):

* tensors appear in kernel read order (``pack_weights.py:28-47``),
* every tensor starts on a 4 KiB boundary (``pack_weights.py:25,71-74``),
* an int8 tensor is its row-major ``[out, in]`` payload followed at once by
  ``[out]`` little-endian fp32 row scales (``pack_weights.py:76-84``),
* an fp32 tensor is written raw (``pack_weights.py:85-89``),
* a JSON manifest (``pack_weights.py:93-101``) and the flat text index read by
  the C++ side (``scripts/emit_weight_index.py:1-22``) describe it.

Which tensors are int8 follows ``golden/quant.py:22-40`` and the per-row
symmetric quantiser is ``golden/quant.py:43-49``.  The random draw is the
pinned generator of the benchmark configs: ``default_rng(seed)`` walked in read order, each
tensor ``standard_normal(shape, float32) * 0.02``.
"""

from __future__ import annotations

import json
import os
import hashlib

import numpy as np

ALIGN = 4096

# Text config of Qwen3.5-0.8B: the values of the reference manifest's
# "config" block (artifacts/qwen35_int8.manifest.json) and hls/src/types.hpp:19-47.
_LAYER_TYPES = (["linear_attention"] * 3 + ["full_attention"]) * 6

QWEN35_08B = {
    "hidden_size": 1024,
    "num_hidden_layers": 24,
    "layer_types": list(_LAYER_TYPES),
    "head_dim": 256,
    "num_attention_heads": 8,
    "num_key_value_heads": 2,
    "intermediate_size": 3584,
    "vocab_size": 248320,
    "rms_norm_eps": 1e-06,
    "linear_num_value_heads": 16,
    "linear_num_key_heads": 16,
    "linear_key_head_dim": 128,
    "linear_value_head_dim": 128,
    "linear_conv_kernel_dim": 4,
    "rope_parameters": {
        "mrope_interleaved": True,
        "mrope_section": [11, 11, 10],
        "rope_type": "default",
        "rope_theta": 10000000,
        "partial_rotary_factor": 0.25,
    },
}

# Names whose 2-D tensors are stored int8 (golden/quant.py:22-34).
INT8_SUFFIXES = (
    "in_proj_qkv.weight", "in_proj_z.weight", "linear_attn.out_proj.weight",
    "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight",
    "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
    "self_attn.o_proj.weight", "embed_tokens.weight",
)


def model_config() -> dict:
    """A fresh copy of the text config (the dict shape golden/model.py reads)."""
    return json.loads(json.dumps(QWEN35_08B))


def is_int8(name: str, shape) -> bool:
    return len(shape) == 2 and name.endswith(INT8_SUFFIXES)


def tensor_order(cfg: dict) -> list[str]:
    """Tensor names in the order one decode token reads them.

    Same sequence as pack_weights.read_order (scripts/pack_weights.py:28-47):
    per layer the input norm, the mixer's tensors, the post norm, the three MLP
    matrices; then the final norm and the tied embedding/head.
    """
    names: list[str] = []
    for li, kind in enumerate(cfg["layer_types"]):
        pre = f"layers.{li}"
        names.append(pre + ".input_layernorm.weight")
        if kind == "linear_attention":
            m = pre + ".linear_attn."
            names.extend(m + s for s in ("in_proj_qkv.weight", "in_proj_z.weight",
                                         "in_proj_b.weight", "in_proj_a.weight",
                                         "conv1d.weight", "A_log", "dt_bias",
                                         "norm.weight", "out_proj.weight"))
        else:
            m = pre + ".self_attn."
            names.extend(m + s for s in ("q_proj.weight", "k_proj.weight", "v_proj.weight",
                                         "q_norm.weight", "k_norm.weight", "o_proj.weight"))
        names.append(pre + ".post_attention_layernorm.weight")
        names.extend(pre + ".mlp." + s for s in ("gate_proj.weight", "up_proj.weight",
                                                 "down_proj.weight"))
    names.extend(["norm.weight", "embed_tokens.weight"])
    return names


def tensor_shapes(cfg: dict) -> dict[str, tuple]:
    """Shape of every text-decoder tensor, as in the HF checkpoint."""
    d = cfg["hidden_size"]
    ffn = cfg["intermediate_size"]
    nh, nkv, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    lh = cfg["linear_num_value_heads"]
    lk, lv = cfg["linear_key_head_dim"], cfg["linear_value_head_dim"]
    key_dim = lk * cfg["linear_num_key_heads"]
    val_dim = lv * lh
    conv_dim = 2 * key_dim + val_dim
    shapes: dict[str, tuple] = {}
    for li, kind in enumerate(cfg["layer_types"]):
        pre = f"layers.{li}"
        shapes[pre + ".input_layernorm.weight"] = (d,)
        shapes[pre + ".post_attention_layernorm.weight"] = (d,)
        if kind == "linear_attention":
            m = pre + ".linear_attn."
            shapes[m + "in_proj_qkv.weight"] = (conv_dim, d)
            shapes[m + "in_proj_z.weight"] = (val_dim, d)
            shapes[m + "in_proj_b.weight"] = (lh, d)
            shapes[m + "in_proj_a.weight"] = (lh, d)
            shapes[m + "conv1d.weight"] = (conv_dim, 1, cfg["linear_conv_kernel_dim"])
            shapes[m + "A_log"] = (lh,)
            shapes[m + "dt_bias"] = (lh,)
            shapes[m + "norm.weight"] = (lv,)
            shapes[m + "out_proj.weight"] = (d, val_dim)
        else:
            m = pre + ".self_attn."
            shapes[m + "q_proj.weight"] = (nh * hd * 2, d)
            shapes[m + "k_proj.weight"] = (nkv * hd, d)
            shapes[m + "v_proj.weight"] = (nkv * hd, d)
            shapes[m + "q_norm.weight"] = (hd,)
            shapes[m + "k_norm.weight"] = (hd,)
            shapes[m + "o_proj.weight"] = (d, nh * hd)
        shapes[pre + ".mlp.gate_proj.weight"] = (ffn, d)
        shapes[pre + ".mlp.up_proj.weight"] = (ffn, d)
        shapes[pre + ".mlp.down_proj.weight"] = (d, ffn)
    shapes["norm.weight"] = (d,)
    shapes["embed_tokens.weight"] = (cfg["vocab_size"], d)
    return shapes


def quantize_rows(w: np.ndarray):
    """Symmetric per-output-row int8: returns (q int8 [out,in], scale fp32 [out]).

    Arithmetic of golden/quant.py:43-49: scale = amax/127 (1.0 for an all-zero
    row), q = clip(rint(w/scale), -127, 127), all in float32.
    """
    if w.ndim != 2:
        raise ValueError("quantize_rows wants a 2-D [out, in] matrix")
    amax = np.max(np.abs(w), axis=1)
    scale = np.where(amax > 0, amax / 127.0, 1.0).astype(np.float32)
    q = np.clip(np.rint(w / scale[:, None]), -127, 127).astype(np.int8)
    return q, scale


def layout(cfg: dict) -> dict:
    """Manifest for the packed blob (offsets depend on shapes only)."""
    shapes = tensor_shapes(cfg)
    ents, off = [], 0
    for name in tensor_order(cfg):
        shp = shapes[name]
        off += (-off) % ALIGN
        n = int(np.prod(shp))
        ent = {"name": name, "shape": list(shp), "offset": off}
        if is_int8(name, shp):
            ent.update(dtype="int8", nbytes=n, scale_offset=off + n, scale_nbytes=4 * shp[0])
            off += n + 4 * shp[0]
        else:
            ent.update(dtype="fp32", nbytes=4 * n)
            off += 4 * n
        ents.append(ent)
    keep = ("hidden_size", "num_hidden_layers", "layer_types", "head_dim",
            "num_attention_heads", "num_key_value_heads", "intermediate_size",
            "vocab_size", "rms_norm_eps", "linear_num_value_heads",
            "linear_key_head_dim", "linear_value_head_dim",
            "linear_conv_kernel_dim", "rope_parameters")
    return {"config": {k: cfg[k] for k in keep}, "align": ALIGN, "total_bytes": off,
            "tensors": ents}


def index_lines(manifest: dict) -> list[str]:
    """Flat index, one line per tensor: name off nbytes dtype scale_off scale_nbytes out in.

    Field meaning of scripts/emit_weight_index.py:1-22 (dtype 1 = int8, 0 = fp32;
    out/in are the first two dims, 0 when absent).
    """
    lines = []
    for t in manifest["tensors"]:
        sh = t["shape"]
        lines.append("%s %d %d %d %d %d %d %d" % (
            t["name"], t["offset"], t["nbytes"], 1 if t["dtype"] == "int8" else 0,
            t.get("scale_offset", 0), t.get("scale_nbytes", 0),
            sh[0] if len(sh) > 0 else 0, sh[1] if len(sh) > 1 else 0))
    return lines


def cache_dir() -> str:
    d = os.environ.get("QWEN_B200_CACHE", "/tmp/qwen_b200_cache")
    os.makedirs(d, exist_ok=True)
    return d


def write_blob(path: str, seed: int = 1234, cfg: dict | None = None, std: float = 0.02) -> dict:
    """Write a random-init blob + ``.manifest.json`` + ``.idx`` beside it.

    Returns the manifest.  Deterministic in ``seed``.
    """
    cfg = cfg or model_config()
    man = layout(cfg)
    shapes = tensor_shapes(cfg)
    rng = np.random.default_rng(seed)
    tmp = path + ".partial"
    with open(tmp, "wb") as f:
        for ent in man["tensors"]:
            f.seek(ent["offset"])
            w = rng.standard_normal(shapes[ent["name"]], np.float32) * std
            if ent["dtype"] == "int8":
                q, s = quantize_rows(w)
                f.write(q.tobytes())
                f.write(s.astype("<f4").tobytes())
            else:
                f.write(w.astype("<f4").tobytes())
        f.truncate(man["total_bytes"])
    os.replace(tmp, path)
    base = os.path.splitext(path)[0]
    with open(base + ".manifest.json", "w") as f:
        json.dump(man, f, indent=1)
    with open(base + ".idx", "w") as f:
        f.write("\n".join(index_lines(man)) + "\n")
    return man


def ensure_blob(seed: int = 1234) -> str:
    """Path of the cached random-init blob for ``seed``, writing it on first use."""
    path = os.path.join(cache_dir(), f"qwen35_08b_rand{seed}.bin")
    base = os.path.splitext(path)[0]
    man = layout(model_config())
    ok = (os.path.exists(path) and os.path.getsize(path) == man["total_bytes"]
          and os.path.exists(base + ".idx") and os.path.exists(base + ".manifest.json"))
    if not ok:
        write_blob(path, seed)
    return path


def index_path(blob_path: str) -> str:
    return os.path.splitext(blob_path)[0] + ".idx"


def manifest_path(blob_path: str) -> str:
    return os.path.splitext(blob_path)[0] + ".manifest.json"


class Blob:
    """Read-only numpy view of a packed blob (int8 payload + scales, fp32 tensors)."""

    def __init__(self, path: str):
        self.path = path
        with open(manifest_path(path)) as f:
            self.manifest = json.load(f)
        self.mm = np.memmap(path, dtype=np.uint8, mode="r")
        self.ents = {t["name"]: t for t in self.manifest["tensors"]}

    def int8(self, name: str):
        t = self.ents[name]
        q = np.frombuffer(self.mm, np.int8, t["nbytes"], t["offset"]).reshape(t["shape"])
        s = np.frombuffer(self.mm, "<f4", t["shape"][0], t["scale_offset"])
        return q, s

    def fp32(self, name: str) -> np.ndarray:
        t = self.ents[name]
        return np.frombuffer(self.mm, "<f4", t["nbytes"] // 4, t["offset"]).reshape(t["shape"])

    def fake_quant(self) -> dict[str, np.ndarray]:
        """fp32 weight dict with int8 tensors dequantised (q * scale per row).

        This is what golden/quant.py:56-76 hands the golden decoder.
        """
        out = {}
        for name, t in self.ents.items():
            if t["dtype"] == "int8":
                q, s = self.int8(name)
                out[name] = q.astype(np.float32) * s[:, None]
            else:
                out[name] = np.array(self.fp32(name))
        return out

    def digest(self) -> str:
        h = hashlib.sha256()
        step = 1 << 24
        for i in range(0, len(self.mm), step):
            h.update(self.mm[i:i + step])
        return h.hexdigest()


def warm_state_arrays(T: int, seed: int, rec_std: float = 0.1, kv_std: float = 1.0, n_lin: int = 18,
                      n_full: int = 6, lh: int = 16, lk: int = 128, lv: int = 128, convd: int = 6144,
                      conv_k: int = 4, nkv: int = 2, hd: int = 256):
    """Warm-start decode state of the W8A8 and long-context configs: DeltaNet
    states N(0, rec_std), conv history zero, T cached positions of K (after
    RoPE) and V drawn N(0, kv_std), pos = T.  Drawn from default_rng(seed) in
    the order rec, then per attention layer K then V (the order the parity
    fixtures were generated with).  Returns a simple namespace with conv, rec,
    kc, vc (lists of [T, nkv, hd]) and pos, as Decoder.import_state takes."""
    from types import SimpleNamespace
    f32 = np.float32
    rng = np.random.default_rng(seed)
    rec = rng.standard_normal((n_lin, lh, lk, lv), f32) * f32(rec_std)
    kc, vc = [], []
    for _ in range(n_full):
        kc.append(rng.standard_normal((T, nkv, hd), f32) * f32(kv_std))
        vc.append(rng.standard_normal((T, nkv, hd), f32) * f32(kv_std))
    return SimpleNamespace(conv=np.zeros((n_lin, convd, conv_k), f32), rec=rec, kc=kc, vc=vc, pos=T)
