"""Tensor-parallel decode over torch.distributed: one process and one GPU per rank.

torch.distributed is only the plumbing here: it carries every rank's 64-byte
exchange-buffer handle at set-up and, when asked, the ranks' logit slices.  The
per-token exchanges (the hidden-vector sums of the row-parallel projections and
the argmax) run inside the decode kernel over NVLink.

Every rank must make the same calls in the same order, as with collectives.
"""

from __future__ import annotations

import numpy as np
import torch.distributed as dist

from . import api


class TPDecoder:
    """Rank `dist.get_rank(group)` of a tensor-parallel decoder."""

    def __init__(self, blob_path: str, index_path: str | None = None, device: int | None = None,
                 max_ctx: int = 4096, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        dev = self.rank if device is None else int(device)
        self.dec = api.Decoder(blob_path, index_path, device=dev, max_ctx=max_ctx,
                               tp_rank=self.rank, tp_world=self.world)
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, self.dec.tp_handle(), group=group)
            self.dec.tp_connect(handles)
        # the ranks' kernels wait on each other with a 2 s bound: start together
        dist.barrier(group)

    def close(self):
        self.dec.close()

    def reset(self):
        self.dec.reset()

    def import_state(self, st):
        self.dec.import_state(st)

    def decode_step(self, tok: int, want_logits: bool = True, sync: bool = True):
        """(argmax, full logits or None).  With want_logits the ranks' vocab
        slices are gathered on every rank."""
        if sync:
            dist.barrier(self.group)
        am, lg = self.dec.decode_step(tok, want_logits=want_logits)
        if not want_logits or self.world == 1:
            return am, lg
        lo, hi = self.dec.vocab_range
        parts = [None] * self.world
        dist.all_gather_object(parts, (lo, hi, lg[lo:hi].copy()), group=self.group)
        full = np.empty_like(lg)
        for a, b, v in parts:
            full[a:b] = v
        return am, full

    def generate(self, prompt, n_new: int, sync: bool = True):
        """Prefill + greedy decode on every rank; (ids, device seconds of the decode steps)."""
        if sync:
            dist.barrier(self.group)
        return self.dec.generate(prompt, n_new)
