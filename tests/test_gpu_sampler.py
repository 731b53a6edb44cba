"""Device sampling (mlb_sample, mlb_decode_sample) against the reference's own
MiniSampler (src/sampler.cc), recorded in tests/golden/sampler.json and live
through oracle/_ref.

The generator is bit-exact (same MT19937 words); the softmax sums differ from
the reference's sequential float loop only in rounding, so an id may differ
only where the uniform draw lies within that rounding of a candidate
boundary. Each mismatch is checked to be such a case, from the draw itself
(numpy's legacy RandomState is the same MT19937) and a float64 evaluation of
the reference's candidate order and running sums."""
import json
import os
import sys

import numpy as np
import pytest

import mini_llama_b200 as mlb

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from sampler_cases import CASES, logits_rows  # noqa: E402

pytestmark = pytest.mark.gpu

BOUNDARY_TOL = 1e-4   # |r - running sum| that rounding of the sums can flip
MAX_FLIPS = 2         # such boundary cases tolerated per case


def golden():
    with open(os.path.join(HERE, "golden", "sampler.json")) as f:
        return json.load(f)


def uniform_draws(seed, n):
    """The reference's uniform_real_distribution<float>(0, 1) draws."""
    u = np.random.RandomState(seed).randint(0, 2**32, size=n, dtype=np.uint32)
    r = u.astype(np.float32) * np.float32(2.0**-32)
    return np.minimum(r, np.float32(np.nextafter(np.float32(1), np.float32(0))))


def candidates(row, temperature, top_k):
    """Candidate ids in the reference's order and their float64 running sums."""
    n = row.size
    if top_k > 1:
        k = min(top_k, n)
        order = np.lexsort((np.arange(n), -row.astype(np.float64)))[:k]
    else:
        order = np.arange(n)
    v = row[order].astype(np.float64)
    p = np.exp((v - v.max()) / temperature)
    return order, np.cumsum(p / p.sum())


def is_greedy(case):
    return case["temperature"] < 1e-6 or case["top_k"] == 1


def check_ids(case, rows, got, want, draws):
    flips = 0
    for i, (g, w) in enumerate(zip(got, want)):
        if g == w:
            continue
        assert not is_greedy(case), (case["name"], i, g, w)
        order, cum = candidates(rows[i], case["temperature"], case["top_k"])
        pos = {int(c): j for j, c in enumerate(order)}
        j = min(pos[g], pos[w])  # the running sum where the two choices part
        assert abs(float(draws[i]) - cum[j]) < BOUNDARY_TOL, (case["name"], i, g, w)
        flips += 1
    assert flips <= MAX_FLIPS, (case["name"], flips)


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_device_sampler_matches_reference(cuda, case):
    torch = pytest.importorskip("torch")
    want = golden()[case["name"]]
    rows = logits_rows(case)
    s = mlb.Sampler(case["seed"])
    dev = torch.from_numpy(rows).cuda()
    got = [s.sample(dev[i].data_ptr(), case["n"], case["temperature"], case["top_k"])
           for i in range(len(rows))]
    s.close()
    check_ids(case, rows, got, want, uniform_draws(case["seed"], len(rows)))


def test_device_sampler_matches_live_reference(cuda, ref):
    """The same against the reference library itself on fresh rows."""
    torch = pytest.importorskip("torch")
    case = dict(name="live", seed=31, temperature=0.7, top_k=64, n=50000, scale=2.5, draws=40)
    rows = logits_rows(case)
    rs = ref.sampler(case["seed"])
    want = [rs.sample(r, case["temperature"], case["top_k"]) for r in rows]
    s = mlb.Sampler(case["seed"])
    dev = torch.from_numpy(rows).cuda()
    got = [s.sample(dev[i].data_ptr(), case["n"], case["temperature"], case["top_k"])
           for i in range(len(rows))]
    check_ids(case, rows, got, want, uniform_draws(case["seed"], len(rows)))


def test_device_sampler_errors(cuda):
    """The reference's checks and messages; a rejected call draws nothing."""
    torch = pytest.importorskip("torch")
    x = torch.zeros(100, device="cuda")
    s = mlb.Sampler(5)
    with pytest.raises(mlb.MlbError, match="cannot sample from empty logits"):
        s.sample(x.data_ptr(), 0, 1.0, 0)
    with pytest.raises(mlb.MlbError, match="top_k must be non-negative"):
        s.sample(x.data_ptr(), 100, 1.0, -1)
    with pytest.raises(mlb.MlbError, match="temperature must be finite and non-negative"):
        s.sample(x.data_ptr(), 100, -0.5, 0)
    with pytest.raises(mlb.MlbError, match="temperature must be finite and non-negative"):
        s.sample(x.data_ptr(), 100, float("nan"), 0)
    big = torch.zeros(10000, device="cuda")
    with pytest.raises(mlb.MlbError, match="top_k above 4096"):
        s.sample(big.data_ptr(), 10000, 1.0, 5000)
    bad = torch.zeros(100, device="cuda")
    bad[37] = float("inf")
    with pytest.raises(mlb.MlbError, match="logits must be finite"):
        s.sample(bad.data_ptr(), 100, 1.0, 0)
    # the first accepted draw is still the stream's first word: equal logits of
    # two candidates pick 0 exactly when r < 0.5
    two = torch.zeros(2, device="cuda")
    r = uniform_draws(5, 1)[0]
    assert s.sample(two.data_ptr(), 2, 1.0, 0) == (0 if r < 0.5 else 1)


def test_decode_sample_matches_reference_sampler(cuda, ref):
    """mlb_decode_sample on a golden small model: every step's id is the
    reference sampler's choice on that step's logits (teacher-forced replay of
    the device ids through mlb_forward_token), with the same seed; and at
    temperature 0 it is decode_greedy."""
    from mini_llama_b200 import configs as C

    with open(os.path.join(HERE, "golden", "golden.json")) as f:
        mt = json.load(f)["small_q4_1_neox_bias"]
    model = mlb.CudaModel(mt["config"]).synthesize(C.Q4_1, 5, with_bias=True)
    steps, t0 = 24, 9
    for kwargs in (dict(temperature=0.9, top_k=0), dict(temperature=1.2, top_k=20)):
        a = model.context()
        s = mlb.Sampler(77)
        ids = a.decode_sample(s, t0, 0, steps, **kwargs)
        b = model.context()
        rs = ref.sampler(77)
        tok, want, rows = t0, [], []
        for pos in range(steps):
            lg = b.forward_token(tok, pos)
            rows.append(lg)
            want.append(rs.sample(lg, kwargs["temperature"], kwargs["top_k"]))
            tok = ids[pos]  # follow the device's ids
        case = dict(name=str(kwargs), **kwargs)
        check_ids(case, np.stack(rows), ids, want, uniform_draws(77, steps))
    a = model.context()
    g = model.context()
    assert a.decode_sample(mlb.Sampler(3), t0, 0, steps, 0.0, 0) == g.decode_greedy(t0, 0, steps)
