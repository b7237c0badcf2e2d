"""Helpers shared by the parity tests: fixture loading and logits comparison."""

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
VOCAB = 248320
# the fixed logit indices stored in the fixtures (tests/golden/make_golden.py)
SAMPLE_IDX = np.sort(np.random.default_rng(7).choice(VOCAB, 4096, replace=False))

# fp32 logits parity bar of the build: max |ours - golden| over the stored
# samples and the top-16, relative to the golden's max |logit|.
LOGIT_RTOL = 1e-4


def fixture(name):
    return np.load(os.path.join(GOLDEN, name))


def logits_close(lg, fx, prefix, rtol=LOGIT_RTOL):
    """Compare a full logits vector with a stored digest; returns the relative error."""
    ref = fx[prefix + "_sample"]
    top_i = fx[prefix + "_top_idx"]
    top_v = fx[prefix + "_top_val"]
    scale = float(fx[prefix + "_absmax"])
    err = max(np.abs(lg[SAMPLE_IDX] - ref).max(), np.abs(lg[top_i] - top_v).max()) / scale
    return float(err)
