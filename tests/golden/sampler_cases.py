"""Seeded cases for MiniSampler::Sample (src/sampler.cc:172-183), shared by
make_sampler_golden.py (which records the reference's ids) and the sampler
tests (which regenerate the same logits rows). Each case is a sampler seed,
the sampling parameters and `draws` logits rows of length n drawn from a
seeded normal distribution times `scale` (optionally rounded to integers so
that many logits tie)."""
import numpy as np

CASES = [
    # temperature over every logit (top_k 0), 7B vocabulary
    dict(name="temp_all_32000", seed=7, temperature=0.8, top_k=0, n=32000, scale=3.0, draws=48),
    # top-k at the usual sizes
    dict(name="topk40_32000", seed=7, temperature=1.0, top_k=40, n=32000, scale=3.0, draws=48),
    dict(name="topk2_1000", seed=3, temperature=1.3, top_k=2, n=1000, scale=1.0, draws=48),
    # the largest device top-k on the 72B vocabulary
    dict(name="topk4096_152064", seed=11, temperature=0.5, top_k=4096, n=152064, scale=2.0,
         draws=12),
    # greedy forms: no draw is taken
    dict(name="greedy_t0_128256", seed=5, temperature=0.0, top_k=0, n=128256, scale=2.0,
         draws=8),
    dict(name="greedy_tiny_t", seed=9, temperature=1e-7, top_k=50, n=5000, scale=2.0, draws=8),
    dict(name="greedy_k1", seed=13, temperature=2.0, top_k=1, n=5000, scale=2.0, draws=8),
    # integer logits: ties inside and at the edge of the top-k set
    dict(name="ties_topk100", seed=17, temperature=1.0, top_k=100, n=4096, scale=2.0,
         draws=48, integer=True),
    # top_k above n is clamped to n
    dict(name="topk_clamped", seed=19, temperature=0.9, top_k=50, n=10, scale=1.0, draws=48),
    # more draws than one MT19937 state (624 words): the regeneration step
    dict(name="long_stream", seed=23, temperature=1.0, top_k=0, n=64, scale=1.0, draws=700),
]


def logits_rows(case):
    rng = np.random.default_rng(1000 + case["seed"] * 7 + case["n"])
    rows = rng.standard_normal((case["draws"], case["n"]), dtype=np.float32) * np.float32(
        case["scale"])
    if case.get("integer"):
        rows = np.round(rows)
    return rows.astype(np.float32)
