"""Decode-step parity on the GPU: the full ForwardToken path through the C ABI
against the reference CPU path's golden outputs (tests/golden, generated from
the reference itself) and the CPU oracle.

Bar: greedy token ids bit-exact; logits within max-abs
2e-3 per step. Attention runs in CPU-compatible mode (the reference CPU path's
V sum, src/forward.cc:518) so greedy parity is against the reference itself.
"""
import json

import numpy as np
import pytest

import mini_llama_b200 as mlb
from mini_llama_b200 import configs as C
from tests.conftest import golden_path

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3
README_TOKENS = [23, 58, 36] + [59] * 61  # README.md:297
# how a decode step runs: the persistent step kernel, or one kernel per op
PATHS = ["step", "per_op"]


def meta():
    with open(golden_path("golden.json")) as f:
        return json.load(f)


def gpu_model(cfg, weights, **kw):
    m = mlb.CudaModel(cfg, **kw)
    m.load(weights)
    return m


def make_ctx(model, path, mode=mlb.ATTN_CPU_COMPAT):
    ctx = model.context(mode, step_kernel=(path == "step"))
    assert ctx.step_kernel() == (path == "step")
    if path == "step":
        assert ctx.kernels_per_step() == 1
    return ctx


def greedy(ctx, prompt, steps, teacher=None):
    logits, toks = [], []
    tok = prompt[0]
    for pos in range(len(prompt) + steps):
        lg = ctx.forward_token(tok, pos)
        logits.append(lg)
        toks.append(int(np.argmax(lg)))
        nxt = teacher[pos] if teacher is not None else toks[-1]
        tok = prompt[pos + 1] if pos + 1 < len(prompt) else nxt
    return np.stack(logits), toks


def readme_weights():
    g = np.load(golden_path("tiny_readme.npz"))
    ws = []
    for key in g.files:
        if key.startswith("w"):
            parts = key[1:].split("_")
            kind, layer = int(parts[0]), (int(parts[1]) if len(parts) > 1 else -1)
            arr = g[key]
            ws.append((kind, layer, C.F32, arr.shape[0], arr.shape[1], arr))
    return g, ws


def test_readme_model_greedy_tokens(cuda):
    g, ws = readme_weights()
    cfg = meta()["tiny_readme"]["config"]
    ctx = gpu_model(cfg, ws).context()
    prompt = [int(t) for t in g["prompt"]]
    logits, toks = greedy(ctx, prompt, 64)
    assert toks[len(prompt) - 1:len(prompt) - 1 + 64] == README_TOKENS
    assert np.abs(logits - g["logits"]).max() <= LOGIT_TOL


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("name", ["small_q4_0_gqa", "small_q4_1_neox_bias", "small_q8_0_ragged"])
def test_small_models_vs_reference(cuda, name, path):
    mt = meta()[name]
    g = np.load(golden_path(f"{name}.npz"))
    qtype = {v: k for k, v in C.QTYPE_NAMES.items()}[mt["qtype"]]
    ws = list(C.host_weights(mt["config"], qtype, mt["seed"], mt["bias"]))
    model = gpu_model(mt["config"], ws)
    prompt = [int(t) for t in g["prompt"]]
    steps = len(g["tokens"]) - len(prompt)
    gold = [int(t) for t in g["tokens"]]
    # teacher-forced: every step sees the reference's token
    logits, toks = greedy(make_ctx(model, path), prompt, steps, teacher=gold)
    err = np.abs(logits - g["logits"]).max(axis=1)
    assert err.max() <= LOGIT_TOL, err
    # free-running greedy: token ids bit-exact
    _, toks2 = greedy(make_ctx(model, path), prompt, steps)
    assert toks2 == gold


@pytest.mark.parametrize("path", PATHS)
def test_tiny_config_greedy_parity(cuda, path):
    """Tiny LLaMA (dim 288, 6 layers, vocab 32000, Q8_0): 16 prompt ids then 128
    greedy steps, token ids bit-exact against the reference CPU path."""
    mt = meta()["tiny_q8_0"]
    g = np.load(golden_path("tiny_q8_0.npz"))
    model = mlb.CudaModel(C.TINY).synthesize(C.Q8_0, mt["seed"])
    prompt = [int(t) for t in g["prompt"]]
    logits, toks = greedy(make_ctx(model, path), prompt, 128)
    gold = [int(t) for t in g["tokens"]]
    if toks != gold:
        i = next(i for i, (a, b) in enumerate(zip(toks, gold)) if a != b)
        pytest.fail(f"first greedy mismatch at step {i}: {toks[i]} vs {gold[i]}, "
                    f"reference top-2 margin {g['margins'][i]:.2e}")
    for i, s in enumerate(g["logit_steps"]):
        assert np.abs(logits[s] - g["logits"][i]).max() <= LOGIT_TOL
    # the on-device greedy loop (one graph launch per step) gives the same ids
    ctx = make_ctx(model, path)
    for pos, t in enumerate(prompt[:-1]):
        ctx.forward_token(t, pos)
    dev = ctx.decode_greedy(prompt[-1], len(prompt) - 1, 129)
    assert dev == gold[len(prompt) - 1:]


def test_device_synthesis_equals_host_weights(cuda):
    cfg, qtype = meta()["small_q4_1_neox_bias"]["config"], C.Q4_1
    ws = list(C.host_weights(cfg, qtype, 21, True))
    a = gpu_model(cfg, ws).context()
    b = mlb.CudaModel(cfg).synthesize(qtype, 21, with_bias=True).context()
    for pos, tok in enumerate([3, 99, 512, 7]):
        np.testing.assert_array_equal(a.forward_token(tok, pos), b.forward_token(tok, pos))


def test_forward_validation_errors(cuda):
    cfg = meta()["small_q8_0_ragged"]["config"]
    model = mlb.CudaModel(cfg).synthesize(C.Q8_0, 1)
    ctx = model.context()
    with pytest.raises(mlb.MlbRangeError, match="token id out of range"):
        ctx.forward_token(cfg["vocab_size"], 0)
    with pytest.raises(mlb.MlbRangeError, match="position out of range"):
        ctx.forward_token(0, cfg["max_seq_len"])
    with pytest.raises(mlb.MlbError):
        mlb.CudaModel(dict(cfg, n_kv_heads=3))
    m2 = mlb.CudaModel(cfg)
    with pytest.raises(mlb.MlbError, match="missing uploaded weight"):
        m2.finalize()
    with pytest.raises(mlb.MlbError, match="shape mismatch"):
        m2.set_weight(C.W_WQ, 0, C.Q8_0, 7, 160, np.zeros(7 * 5 * 34, np.uint8))


def test_standard_attention_mode_differs_only_in_v_sum(cuda, port):
    cfg = meta()["small_q4_0_gqa"]["config"]
    model = mlb.CudaModel(cfg).synthesize(C.Q4_0, 2)
    a = model.context(mlb.ATTN_CPU_COMPAT)
    b = model.context(mlb.ATTN_STANDARD)
    la, lb = a.forward_token(5, 0), b.forward_token(5, 0)
    assert not np.array_equal(la, lb)  # pos 0: the CPU path sums no V row at all


@pytest.mark.parametrize("path", PATHS)
def test_long_context_step(cuda, port, path):
    """A step deep into the context (many attention splits) against the oracle."""
    cfg = dict(meta()["small_q4_0_gqa"]["config"], max_seq_len=1024)
    ws = list(C.host_weights(cfg, C.Q4_0, 4))
    gm = gpu_model(cfg, ws)
    pm = port.model(cfg)
    for kind, layer, qtype, rows, cols, arr in ws:
        pm.set_weight(kind, layer, qtype, rows, cols, arr)
    ctx = make_ctx(gm, path)
    rng = np.random.default_rng(0)
    toks = rng.integers(0, cfg["vocab_size"], 700)
    for pos, t in enumerate(toks):
        lg = ctx.forward_token(int(t), pos)
        lp = pm.forward_token(int(t), pos)
        if pos % 97 == 0 or pos == len(toks) - 1:
            assert np.abs(lg - lp).max() <= LOGIT_TOL, pos


@pytest.mark.parametrize("mode", [mlb.ATTN_CPU_COMPAT, mlb.ATTN_STANDARD])
@pytest.mark.parametrize("name", ["small_q4_0_gqa", "small_q4_1_neox_bias", "small_q8_0_ragged"])
def test_step_kernel_matches_per_op_path(cuda, name, mode):
    """Both step paths, both attention modes: same greedy ids, logits within the
    bar (the projections are the same instructions; attention is summed in a
    different order)."""
    mt = meta()[name]
    qtype = {v: k for k, v in C.QTYPE_NAMES.items()}[mt["qtype"]]
    model = mlb.CudaModel(mt["config"]).synthesize(qtype, 11, with_bias=mt["bias"])
    a, b = make_ctx(model, "step", mode), make_ctx(model, "per_op", mode)
    tok_a = tok_b = 17
    for pos in range(mt["config"]["max_seq_len"]):
        la, lb = a.forward_token(tok_a, pos), b.forward_token(tok_b, pos)
        assert np.abs(la - lb).max() <= LOGIT_TOL, pos
        tok_a, tok_b = int(np.argmax(la)), int(np.argmax(lb))
        assert tok_a == tok_b, pos


def test_step_kernel_selection(cuda):
    """Quantised single-GPU models default to the step kernel; F32 weights run
    per op, and asking for the step kernel there names the reason."""
    mt = meta()["small_q4_0_gqa"]
    model = mlb.CudaModel(mt["config"]).synthesize(C.Q4_0, 3)
    ctx = model.context()
    assert ctx.step_kernel() and ctx.kernels_per_step() == 1
    ctx.set_step_kernel(False)
    assert not ctx.step_kernel() and ctx.kernels_per_step() > 1
    _, ws = readme_weights()
    f32 = gpu_model(meta()["tiny_readme"]["config"], ws).context()
    assert not f32.step_kernel()
    with pytest.raises(mlb.MlbError, match="not Q4_0/Q4_1/Q8_0"):
        f32.set_step_kernel(True)


def test_step_trace(cuda):
    """The step kernel's phase trace: one traced step gives stamps for 5 phases
    per layer plus lm_head on every CTA, in order; the traced steps decode the
    same ids; a read
    with no step since the last one, tracing on the per-op path, and reading
    with tracing off are refused."""
    mt = meta()["small_q4_0_gqa"]
    model = mlb.CudaModel(mt["config"]).synthesize(C.Q4_0, 3)
    plain = make_ctx(model, "step").decode_greedy(5, 0, 4)
    ctx = make_ctx(model, "step")
    with pytest.raises(mlb.MlbError, match="tracing is off"):
        ctx.step_trace_read()
    ctx.step_trace(True)
    ids, tok = [], 5
    for pos in range(4):
        tok = ctx.decode_greedy(tok, pos, 1)[-1]
        ids.append(tok)
        t = ctx.step_trace_read().astype(np.int64)
        assert t.shape[0] == 5 * mt["config"]["n_layers"] + 1 and t.shape[2] == 2
        assert (t[:, :, 1] >= t[:, :, 0]).all()          # each phase ends after it starts
        assert (t[1:, :, 0] >= t[:-1, :, 1]).all()       # and each CTA's phases in order
    assert ids == plain
    with pytest.raises(mlb.MlbError, match="no whole traced step"):
        ctx.step_trace_read()
    ctx.step_trace(False)
    per_op = make_ctx(model, "per_op")
    with pytest.raises(mlb.MlbError, match="not on the step kernel"):
        per_op.step_trace(True)


def test_step_kernel_decode_greedy_matches_forward(cuda):
    """The on-device greedy loop of the step kernel (position, token and step
    advanced by the kernel itself) against step-by-step host decoding."""
    mt = meta()["small_q4_1_neox_bias"]
    model = mlb.CudaModel(mt["config"]).synthesize(C.Q4_1, 5, with_bias=True)
    a = make_ctx(model, "step")
    host, tok = [], 9
    for pos in range(40):
        tok = int(np.argmax(a.forward_token(tok, pos)))
        host.append(tok)
    b = make_ctx(model, "step")
    assert b.decode_greedy(9, 0, 40) == host


@pytest.mark.parametrize("qtype", [C.Q4_0, C.Q8_0])
def test_step_kernel_two_chunk_groups_matches_per_op_path(cuda, qtype):
    """A hidden size above 16384 inputs splits w_down's K into chunk groups
    (66 chunks: 32 + 32 + 2), and with 256 output tiles (768 group-tiles over
    148 CTAs) many CTA ranges of the step kernel span two group segments whose
    tiles are finished across CTAs (the 72B shape's w_down): greedy ids equal
    and logits within the bar of the per-op path over 12 steps."""
    cfg = dict(vocab_size=512, dim=4096, hidden_dim=16896, n_layers=2, n_heads=32, n_kv_heads=8,
               head_dim=128, max_seq_len=16, rope_theta=10000.0, rms_norm_eps=1e-5, rope_type=0)
    model = mlb.CudaModel(cfg).synthesize(qtype, 5)
    a, b = make_ctx(model, "step"), make_ctx(model, "per_op")
    tok_a = tok_b = 11
    for pos in range(12):
        la, lb = a.forward_token(tok_a, pos), b.forward_token(tok_b, pos)
        assert np.abs(la - lb).max() <= LOGIT_TOL, pos
        tok_a, tok_b = int(np.argmax(la)), int(np.argmax(lb))
        assert tok_a == tok_b, pos
