"""The CPU oracle (oracle/port) pinned against the reference's golden vectors,
its known-answer tests, and (where built) the reference's own code."""
import json

import numpy as np
import pytest

from tests.conftest import golden_path
from mini_llama_b200 import configs as C

README_TOKENS = [23, 58, 36] + [59] * 61  # README.md:297, prompt "hello"


def golden_meta():
    with open(golden_path("golden.json")) as f:
        return json.load(f)


def run_port(port, cfg, weights, prompt, steps, teacher=None):
    m = port.model(cfg)
    for kind, layer, qtype, rows, cols, arr in weights:
        m.set_weight(kind, layer, qtype, rows, cols, arr)
    logits, toks = [], []
    tok = prompt[0]
    for pos in range(len(prompt) + steps):
        lg = m.forward_token(tok, pos)
        logits.append(lg)
        toks.append(int(np.argmax(lg)))
        nxt = teacher[pos] if teacher is not None else toks[-1]
        tok = prompt[pos + 1] if pos + 1 < len(prompt) else nxt
    return np.stack(logits), toks


# ------------------------------------------------------------ known answers

def test_block_layouts():
    # tests/test_quant.cc:7-11, 180-190
    assert C.BLOCK_BYTES == {C.Q8_0: 34, C.Q4_0: 18, C.Q4_1: 20}


def test_q4_1_dequant_known_values(port):
    # tests/test_quant.cc:227-244: d = fp16(0.5), m = fp16(-1), q_i = i | (15-i) << 4
    blk = np.zeros(20, np.uint8)
    blk[0:2] = np.frombuffer(np.uint16(0x3800).tobytes(), np.uint8)
    blk[2:4] = np.frombuffer(np.uint16(0xBC00).tobytes(), np.uint8)
    blk[4:] = [i | ((15 - i) << 4) for i in range(16)]
    out = port.dequant(C.Q4_1, blk, 1, 32)[0]
    want = np.array([-1.0 + 0.5 * i for i in range(16)] + [-1.0 + 0.5 * (15 - i) for i in range(16)],
                    np.float32)
    np.testing.assert_array_equal(out, want)


def test_q4_1_linear_known_value(port):
    # tests/test_quant.cc:246-259: d = 1, m = 0, all nibbles 1, x = 2 -> 64
    blk = np.zeros(20, np.uint8)
    blk[0:2] = np.frombuffer(np.uint16(0x3C00).tobytes(), np.uint8)
    blk[4:] = 0x11
    y = port.linear(C.Q4_1, np.full(32, 2.0, np.float32), blk, 1)
    assert y[0] == 64.0


def test_q8_0_roundtrip_and_zeros(port):
    # tests/test_quant.cc:16-52
    src = (np.arange(32, dtype=np.float32) * np.float32(0.1))[None]
    q = port.quantize(C.Q8_0, src)
    assert q.size == 34
    assert np.abs(port.dequant(C.Q8_0, q, 1, 32) - src).max() < 6e-2
    z = port.quantize(C.Q8_0, np.zeros((1, 64), np.float32))
    assert z.size == 68 and not port.dequant(C.Q8_0, z, 1, 64).any()


def test_q4_0_roundtrip(port):
    src = (np.arange(32, dtype=np.float32) * np.float32(0.1))[None]
    q = port.quantize(C.Q4_0, src)
    assert q.size == 18
    assert np.abs(port.dequant(C.Q4_0, q, 1, 32) - src).max() < 3e-1


def test_fp16_conversion_rounding(port):
    # half-up rounding of the dropped mantissa bits (src/quant.cc:38-47)
    assert port.f32_to_fp16(1.0) == 0x3C00
    assert port.f32_to_fp16(-1.0) == 0xBC00
    assert port.f32_to_fp16(0.5) == 0x3800
    assert port.f32_to_fp16(1e9) == 0x7C00
    assert port.f32_to_fp16(1e-9) == 0x0000
    tie = np.frombuffer(np.uint32(0x3F801000).tobytes(), np.float32)[0]  # 1 + 2^-11
    assert port.f32_to_fp16(float(tie)) == 0x3C01  # rounds up, not to even
    for h in (0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF, 0x8001):
        f = port.fp16_to_f32(h)
        assert np.float16(np.frombuffer(np.uint16(h).tobytes(), np.float16)[0]) == np.float16(f)


def test_attention_cpu_quirk_at_pos0(port):
    # src/forward.cc:518: the V sum stops before pos, so pos 0 gives exactly 0
    rng = np.random.default_rng(0)
    keys = rng.normal(size=(1, 4, 2, 8)).astype(np.float32)
    vals = rng.normal(size=(1, 4, 2, 8)).astype(np.float32)
    q = rng.normal(size=(4, 8)).astype(np.float32)
    assert not port.attention(q, keys, vals, 0, 0, 4, 2, 8).any()
    assert port.attention(q, keys, vals, 0, 0, 4, 2, 8, include_current_v=True).any()


# ------------------------------------------------------------- golden models

def test_readme_tiny_model_tokens(port):
    g = np.load(golden_path("tiny_readme.npz"))
    cfg = golden_meta()["tiny_readme"]["config"]
    weights = []
    for key in g.files:
        if not key.startswith("w"):
            continue
        parts = key[1:].split("_")
        kind, layer = int(parts[0]), (int(parts[1]) if len(parts) > 1 else -1)
        arr = g[key]
        weights.append((kind, layer, C.F32, arr.shape[0], arr.shape[1], arr))
    prompt = [int(t) for t in g["prompt"]]
    logits, toks = run_port(port, cfg, weights, prompt, 64)
    assert toks[len(prompt) - 1:len(prompt) - 1 + 64] == README_TOKENS
    np.testing.assert_array_equal(logits, g["logits"])


@pytest.mark.parametrize("name", ["small_q4_0_gqa", "small_q4_1_neox_bias", "small_q8_0_ragged"])
def test_small_models_match_reference_bits(port, name):
    meta = golden_meta()[name]
    g = np.load(golden_path(f"{name}.npz"))
    cfg = meta["config"]
    qtype = {v: k for k, v in C.QTYPE_NAMES.items()}[meta["qtype"]]
    weights = list(C.host_weights(cfg, qtype, meta["seed"], meta["bias"]))
    prompt = [int(t) for t in g["prompt"]]
    logits, toks = run_port(port, cfg, weights, prompt, len(g["tokens"]) - len(prompt))
    np.testing.assert_array_equal(logits, g["logits"])
    assert toks == [int(t) for t in g["tokens"]]


def test_tiny_q8_0_first_steps_match_reference_bits(port):
    meta = golden_meta()["tiny_q8_0"]
    g = np.load(golden_path("tiny_q8_0.npz"))
    weights = list(C.host_weights(C.TINY, C.Q8_0, meta["seed"]))
    prompt = [int(t) for t in g["prompt"]]
    logits, toks = run_port(port, C.TINY, weights, prompt, 1)
    steps = list(g["logit_steps"])
    for i, s in enumerate(steps):
        if s < len(logits):
            np.testing.assert_array_equal(logits[s], g["logits"][i])
    assert toks == [int(t) for t in g["tokens"][: len(toks)]]


# ---------------------------------------------------- port vs reference code

@pytest.mark.parametrize("qtype", [C.Q8_0, C.Q4_0, C.Q4_1])
@pytest.mark.parametrize("shape", [(5, 13), (32, 64), (17, 65), (9, 288)])
def test_linear_bits_vs_reference(port, ref, qtype, shape):
    rng = np.random.default_rng(shape[0] * 100 + qtype)
    w = rng.normal(0, 0.05, shape).astype(np.float32)
    q = port.quantize(qtype, w)
    if qtype != C.Q4_1:
        np.testing.assert_array_equal(q, ref.quantize(qtype, w))
    np.testing.assert_array_equal(port.dequant(qtype, q, *shape), ref.dequant(qtype, q, *shape))
    x = rng.normal(0, 1, (3, shape[1])).astype(np.float32)
    np.testing.assert_array_equal(port.linear(qtype, x, q, shape[0]),
                                  ref.linear(qtype, x, q, shape[0]))


def test_elementwise_bits_vs_reference(port, ref):
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, 288).astype(np.float32)
    w = rng.normal(1, 0.1, 288).astype(np.float32)
    np.testing.assert_array_equal(port.rmsnorm(x, w, 1e-5), ref.rmsnorm(x, w, 1e-5))
    np.testing.assert_array_equal(port.softmax(x), ref.softmax(x))
    np.testing.assert_array_equal(port.swiglu(x, w), ref.swiglu(x, w))
    assert port.argmax(x) == ref.argmax(x)
    tie = np.array([1.0, 3.0, 3.0, 2.0], np.float32)
    assert port.argmax(tie) == ref.argmax(tie) == 1
    for neox in (0, 1):
        q = rng.normal(size=(6, 48)).astype(np.float32)
        k = rng.normal(size=(2, 48)).astype(np.float32)
        for pos in (0, 1, 37, 255):
            a, b = port.rope(q, k, pos, 10000.0, neox), ref.rope(q, k, pos, 10000.0, neox)
            np.testing.assert_array_equal(a[0], b[0])
            np.testing.assert_array_equal(a[1], b[1])


def test_forward_errors_match_reference(port, ref):
    cfg = golden_meta()["small_q8_0_ragged"]["config"]
    weights = list(C.host_weights(cfg, C.Q8_0, 7))
    pm, rm = port.model(cfg), ref.model(cfg)
    for kind, layer, qtype, rows, cols, arr in weights:
        pm.set_weight(kind, layer, qtype, rows, cols, arr)
        rm.set_weight(kind, layer, qtype, rows, cols, arr)
    for bad_tok, bad_pos in ((-1, 0), (cfg["vocab_size"], 0), (0, cfg["max_seq_len"]), (0, -1)):
        with pytest.raises(IndexError):
            pm.forward_token(bad_tok, bad_pos)
        with pytest.raises(IndexError):
            rm.forward_token(bad_tok, bad_pos)


# ------------------------------------------- reference arm inputs (no project .so)

@pytest.mark.parametrize("qtype,bias", [(C.Q8_0, False), (C.Q4_0, False), (C.Q4_1, True)])
def test_reference_model_synthesis_equals_generator_bytes(ref, qtype, bias):
    """The reference arm builds its model inside oracle/_ref (the seeded
    generator quantised with the reference's own QuantizeToQ80/Q40): its
    logits equal, bit for bit, those of the same model loaded from the GPU
    library's host generator, so both arms decode identical weights."""
    cfg = dict(vocab_size=300, dim=96, hidden_dim=160, n_layers=2, n_heads=4, n_kv_heads=2,
               head_dim=24, max_seq_len=16, rope_theta=10000.0, rms_norm_eps=1e-5,
               rope_type=1 if bias else 0)
    a = ref.model(cfg).synthesize(qtype, 77, bias, threads=3)
    b = ref.model(cfg)
    for kind, layer, qt, rows, cols, arr in C.host_weights(cfg, qtype, 77, bias):
        b.set_weight(kind, layer, qt, rows, cols, arr)
    tok = 5
    for pos in range(4):
        la, lb = a.forward_token(tok, pos), b.forward_token(tok, pos)
        np.testing.assert_array_equal(la.view(np.uint32), lb.view(np.uint32))
        tok = int(np.argmax(la))


def test_reference_kv_fill_is_deterministic(ref):
    cfg = dict(vocab_size=200, dim=64, hidden_dim=96, n_layers=2, n_heads=4, n_kv_heads=4,
               head_dim=16, max_seq_len=32, rope_theta=10000.0, rms_norm_eps=1e-5, rope_type=0)
    outs = []
    for _ in range(2):
        m = ref.model(cfg).synthesize(C.Q4_0, 3)
        m.fill_kv(20, 11)
        outs.append(m.forward_token(7, 20))
    np.testing.assert_array_equal(outs[0], outs[1])
    m = ref.model(cfg).synthesize(C.Q4_0, 3)
    m.fill_kv(20, 12)  # another seed changes the attended context
    assert not np.array_equal(outs[0], m.forward_token(7, 20))
    with pytest.raises(IndexError):
        m.fill_kv(33, 1)


def test_reference_sampler_reproduces_golden(ref):
    """oracle/_ref's MiniSampler (src/sampler.cc) gives the recorded ids."""
    import json
    import os
    import sys

    here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    sys.path.insert(0, here)
    from sampler_cases import CASES, logits_rows

    with open(os.path.join(here, "sampler.json")) as f:
        want = json.load(f)
    for case in CASES:
        s = ref.sampler(case["seed"])
        got = [s.sample(r, case["temperature"], case["top_k"]) for r in logits_rows(case)]
        assert got == want[case["name"]], case["name"]


def test_reference_sampler_uniform_draws(ref):
    """The draw the device sampler restates: uniform_real_distribution<float>
    over std::mt19937 is float(u) / 2^32 of one 32-bit word (numpy's legacy
    RandomState is the same generator). Two equal logits at temperature 1 pick
    index 0 exactly when that draw is below 0.5."""
    import numpy as np

    seed, n = 12345, 2000
    u = np.random.RandomState(seed).randint(0, 2**32, size=n, dtype=np.uint32)
    r = u.astype(np.float32) * np.float32(2.0**-32)
    s = ref.sampler(seed)
    zeros = np.zeros(2, np.float32)
    got = [s.sample(zeros, 1.0, 0) for _ in range(n)]
    assert got == [0 if x < 0.5 else 1 for x in r]


def test_reference_sampler_errors(ref):
    import numpy as np

    s = ref.sampler(1)
    x = np.zeros(8, np.float32)
    for t, k, msg in ((-1.0, 0, "temperature"), (1.0, -2, "top_k"),
                      (float("inf"), 0, "temperature")):
        with pytest.raises(RuntimeError, match=msg):
            s.sample(x, t, k)
    x[3] = np.nan
    with pytest.raises(RuntimeError, match="finite"):
        s.sample(x, 1.0, 0)
