"""Prompt front-end on the B200 backend: the counterpart of the reference's
run_prompt.py (run_prompt.py:35-113) with `decode_step` running on the GPU.

    python -m qwen_fpga_b200.run_prompt --snapshot SNAP --blob qwen.bin -p "Explain FPGAs." -n 80
    python -m qwen_fpga_b200.run_prompt --snapshot SNAP --blob qwen.bin -p "def fib(n):" --raw
    python -m qwen_fpga_b200.run_prompt --synthetic --ids 211227,158170,126925 -n 16

Same flow as the reference: tokenize the prompt (the chat template unless
--raw, run_prompt.py:58-67), feed it, then decode greedily until EOS or -n
tokens, timing only the decode steps (run_prompt.py:80-98).  Differences:
- the prompt goes through every layer in one `qwen_prefill` pass (the chunked
  delta rule) instead of one decode step per token;
- weights are always the int8 blob (the reference's --int8); --w8a8 also
  quantises the activations (ACT_INT8, the reference's --w8a8).  There is no
  fp32-weight path;
- the blob comes from --blob, packed first from --snapshot with
  `qwen_pack_blob` when it does not exist, or --synthetic uses the seeded
  random-init model (token ids only: it has no tokenizer);
- without a tokenizer (no snapshot, or transformers absent) the prompt is
  given as token ids (--ids) and the answer is printed as ids.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np


def parse_ids(text: str) -> list[int]:
    """'1,2, 3' -> [1, 2, 3]; raises ValueError on anything else or on an empty list."""
    ids = [int(t) for t in text.replace(" ", "").split(",") if t != ""]
    if not ids:
        raise ValueError("--ids needs at least one token id")
    return ids


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="python -m qwen_fpga_b200.run_prompt",
                                 description="Run a prompt through Qwen3.5-0.8B on a B200.")
    src = ap.add_mutually_exclusive_group(required=True)
    src.add_argument("-p", "--prompt", help="prompt text (needs --snapshot's tokenizer)")
    src.add_argument("--ids", help="prompt as comma-separated token ids")
    ap.add_argument("-n", "--n_new", type=int, default=64, help="max tokens to generate")
    ap.add_argument("--w8a8", action="store_true", help="int8 activations too (ACT_INT8)")
    ap.add_argument("--raw", action="store_true", help="raw completion; skip the chat template")
    ap.add_argument("--snapshot", help="Hugging Face snapshot directory (config, tokenizer, safetensors)")
    ap.add_argument("--blob", help="packed int8 blob; packed from --snapshot when it does not exist")
    ap.add_argument("--synthetic", action="store_true", help="the seeded random-init model (ids only)")
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--eos", type=int, action="append", default=[], help="extra EOS token id")
    ap.add_argument("--quiet", action="store_true", help="print only the JSON summary")
    return ap


def _tokenizer(snapshot):
    if not snapshot:
        return None
    try:
        from transformers import AutoTokenizer
    except ImportError:
        return None
    return AutoTokenizer.from_pretrained(snapshot)


def _encode(tok, prompt: str, raw: bool) -> list[int]:
    if raw:
        return tok(prompt, return_tensors="np").input_ids[0].tolist()
    enc = tok.apply_chat_template([{"role": "user", "content": prompt}], add_generation_prompt=True,
                                  tokenize=True)
    if not isinstance(enc, (list, tuple, np.ndarray)):   # transformers 5: a BatchEncoding
        enc = enc["input_ids"]
    return np.asarray(enc).reshape(-1).tolist()


def _blob(args) -> str:
    if args.synthetic:
        from . import synth
        return synth.ensure_blob(1234)
    if not args.blob:
        raise SystemExit("give --blob (packed from --snapshot if missing) or --synthetic")
    if not os.path.exists(args.blob):
        if not args.snapshot:
            raise SystemExit(f"{args.blob} does not exist and no --snapshot to pack it from")
        from . import api
        print(f"packing {args.snapshot} -> {args.blob} ...", file=sys.stderr, flush=True)
        api.pack_blob(args.snapshot, args.blob)
    return args.blob


def run(argv=None) -> dict:
    """Parse argv, run the prompt, print as the reference does; returns the
    summary dict (prompt ids, generated ids, timings)."""
    args = build_parser().parse_args(argv)
    from . import api

    tok = _tokenizer(args.snapshot)
    if args.prompt is not None:
        if tok is None:
            raise SystemExit("-p needs a tokenizer (--snapshot with transformers installed); use --ids")
        ids = _encode(tok, args.prompt, args.raw)
    else:
        ids = parse_ids(args.ids)
    eos = set(args.eos)
    if tok is not None and tok.eos_token_id is not None:
        eos.add(int(tok.eos_token_id))
    if args.snapshot and os.path.exists(os.path.join(args.snapshot, "config.json")):
        with open(os.path.join(args.snapshot, "config.json")) as f:
            cfg = json.load(f)
        e = cfg.get("eos_token_id", cfg.get("text_config", {}).get("eos_token_id"))
        for v in (e if isinstance(e, list) else [e]):
            if v is not None:
                eos.add(int(v))

    blob = _blob(args)
    dec = api.Decoder(blob, device=args.device, max_ctx=max(256, len(ids) + args.n_new + 1),
                      act_int8=args.w8a8)
    say = (lambda *a, **k: None) if args.quiet else print
    try:
        say(f"\nprompt      : {args.prompt!r}" if args.prompt is not None else f"\nprompt ids  : {ids}")
        say(f"weights     : int8 blob, {'W8A8 (int8 activations)' if args.w8a8 else 'fp32 activations'}")
        say(f"prompt len  : {len(ids)} tokens\n")
        t0 = time.perf_counter()
        nxt, _ = dec.prefill(ids, want_logits=False)
        t_prefill = time.perf_counter() - t0
        say("answer      : ", end="", flush=True)
        out, t_dec = [], 0.0
        for _ in range(args.n_new):
            if nxt in eos:
                break
            out.append(int(nxt))
            say(tok.decode([nxt]) if tok is not None else f"{nxt} ", end="", flush=True)
            d0 = time.perf_counter()
            nxt, _ = dec.decode_step(nxt, want_logits=False)
            t_dec += time.perf_counter() - d0
        say("\n")
    finally:
        dec.close()
    n_gen = len(out)
    pf_rate = len(ids) / t_prefill if t_prefill else 0.0
    dc_rate = n_gen / t_dec if t_dec else 0.0
    say("--- speed (B200, host wall clock) -------------------------")
    say(f"prefill     : {len(ids):>4} tok in {t_prefill * 1e3:8.2f} ms  {pf_rate:9.1f} tok/s  (one qwen_prefill)")
    say(f"decode      : {n_gen:>4} tok in {t_dec * 1e3:8.2f} ms  {dc_rate:9.1f} tok/s  (qwen_decode_step each)")
    res = {"prompt_ids": ids, "ids": out, "prefill_s": t_prefill, "decode_s": t_dec,
           "prefill_tok_s": pf_rate, "decode_tok_s": dc_rate}
    if args.quiet:
        print(json.dumps(res))
    return res


def main(argv=None) -> int:
    run(argv)
    return 0


if __name__ == "__main__":
    sys.exit(main())
