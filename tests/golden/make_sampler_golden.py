"""Records the reference's sampler ids for tests/golden/sampler_cases.py into
sampler.json, from the reference's own MiniSampler (src/sampler.cc) compiled
into oracle/_ref/libmlref.so (``make -C oracle ref``):

    python tests/golden/make_sampler_golden.py
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

import oracle  # noqa: E402
from sampler_cases import CASES, logits_rows  # noqa: E402


def main():
    ref = oracle.Ref()
    out = {}
    for case in CASES:
        s = ref.sampler(case["seed"])
        ids = [s.sample(row, case["temperature"], case["top_k"]) for row in logits_rows(case)]
        out[case["name"]] = ids
    with open(os.path.join(HERE, "sampler.json"), "w") as f:
        json.dump(out, f)
    print("wrote", len(out), "cases")


if __name__ == "__main__":
    main()
