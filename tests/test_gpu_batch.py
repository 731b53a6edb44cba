"""Batched decode and ForwardBatch (prompt prefill) on the tensor-core GEMM.

Reference behaviour: ForwardBatch (src/batch.cc:35-50) is ForwardToken per
token, in order; several sequences are several MiniLlamaContexts. So:

* ForwardBatch of a prompt gives the last token's logits of the sequential
  ForwardToken loop (CPU oracle and the GPU single-token step), and leaves the
  KV cache such that decoding continues identically;
* a batch of sequences decoded in lockstep gives, per sequence, the greedy ids
  of that sequence decoded alone (the reference CPU path for a subset, the
  single-token GPU step for all), at the full 8B / 72B widths at batch 32.

Bars: greedy ids bit-exact; logits max-abs 2e-3 (BASELINE's parity rule).
"""
import json
import os

import numpy as np
import pytest

import mini_llama_b200 as mlb
from mini_llama_b200 import configs as C
from tests.conftest import golden_path

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3
SEED = 20261201


def meta():
    with open(golden_path("golden.json")) as f:
        return json.load(f)


def port_model(port, cfg, qtype, seed, bias):
    pm = port.model(cfg)
    for kind, layer, qt, rows, cols, arr in C.host_weights(cfg, qtype, seed, bias):
        pm.set_weight(kind, layer, qt, rows, cols, arr)
    return pm


@pytest.mark.parametrize("name", ["small_q4_0_gqa", "small_q4_1_neox_bias", "small_q8_0_ragged"])
def test_forward_batch_prefill_matches_sequential(cuda, port, name):
    mt = meta()[name]
    cfg = mt["config"]
    qtype = {v: k for k, v in C.QTYPE_NAMES.items()}[mt["qtype"]]
    model = mlb.CudaModel(cfg).synthesize(qtype, 31, with_bias=mt["bias"])
    pm = port_model(port, cfg, qtype, 31, mt["bias"])
    rng = np.random.default_rng(5)
    n = min(cfg["max_seq_len"] - 6, 40)
    prompt = [int(t) for t in rng.integers(0, cfg["vocab_size"], n)]
    for pos, t in enumerate(prompt):
        lp = pm.forward_token(t, pos)
    seq = model.context()
    for pos, t in enumerate(prompt):
        ls = seq.forward_token(t, pos)
    bat = model.context()
    lb = bat.forward_batch(prompt, list(range(n)))
    assert np.abs(lb - lp).max() <= LOGIT_TOL
    assert np.abs(lb - ls).max() <= LOGIT_TOL
    assert int(np.argmax(lb)) == int(np.argmax(lp))
    # the KV cache the batch wrote continues the decode like the sequential one
    tok = int(np.argmax(lb))
    for pos in range(n, n + 5):
        la, lc = bat.forward_token(tok, pos), pm.forward_token(tok, pos)
        assert np.abs(la - lc).max() <= LOGIT_TOL, pos
        assert int(np.argmax(la)) == int(np.argmax(lc))
        tok = int(np.argmax(lc))
    # a prompt longer than one 64-row pass, split by the library
    if cfg["max_seq_len"] >= 100:
        long_p = [int(t) for t in rng.integers(0, cfg["vocab_size"], 90)]
        c2 = model.context()
        lb2 = c2.forward_batch(long_p, list(range(90)))
        c3 = model.context()
        for pos, t in enumerate(long_p):
            l3 = c3.forward_token(t, pos)
        assert np.abs(lb2 - l3).max() <= LOGIT_TOL


def test_forward_batch_validation(cuda):
    cfg = meta()["small_q4_0_gqa"]["config"]
    model = mlb.CudaModel(cfg).synthesize(C.Q4_0, 3)
    ctx = model.context()
    with pytest.raises(mlb.MlbError, match="strictly increasing"):
        ctx.forward_batch([1, 2, 3], [0, 2, 1])
    with pytest.raises(mlb.MlbRangeError, match="token id out of range"):
        ctx.forward_batch([1, cfg["vocab_size"]], [0, 1])
    with pytest.raises(mlb.MlbRangeError, match="position out of range"):
        ctx.forward_batch([1], [cfg["max_seq_len"]])
    with pytest.raises(mlb.MlbError, match="empty batch"):
        ctx.forward_batch([], [])


@pytest.mark.parametrize("name", ["small_q4_0_gqa", "small_q4_1_neox_bias", "small_q8_0_ragged"])
def test_batch_decode_matches_independent_sequences(cuda, port, name):
    """5 sequences at different depths and tokens, decoded in lockstep, against
    each sequence decoded alone (CPU oracle and the single-token GPU step)."""
    mt = meta()[name]
    cfg = mt["config"]
    qtype = {v: k for k, v in C.QTYPE_NAMES.items()}[mt["qtype"]]
    model = mlb.CudaModel(cfg).synthesize(qtype, 17, with_bias=mt["bias"])
    pm = port_model(port, cfg, qtype, 17, mt["bias"])
    n_seqs, steps = 5, 8
    depths = [0, 3, 7, 1, 12]
    toks = [3, 77, 150, 9, 200]
    b = mlb.Batch(model, n_seqs)
    for s in range(n_seqs):
        b.fill_kv(s, depths[s], 100 + s)
    got = b.decode_greedy(toks, depths, steps)
    assert got.shape == (steps, n_seqs)
    assert b.kernels_per_step() > 0
    for s in range(n_seqs):
        ctx = model.context()
        ctx.fill_kv(depths[s], 100 + s)
        want = ctx.decode_greedy(toks[s], depths[s], steps)
        assert list(got[:, s]) == want, s
    # logits of one pass against the oracle (sequence 1 of the same state)
    b2 = mlb.Batch(model, 2)
    rng = np.random.default_rng(0)
    pr = [int(t) for t in rng.integers(0, cfg["vocab_size"], 6)]
    for pos, t in enumerate(pr):
        nxt, lg = b2.forward([0, 1], [t, t], [pos, pos], logits=True)
        lp = pm.forward_token(t, pos)
        assert np.abs(lg[1] - lp).max() <= LOGIT_TOL
        assert np.array_equal(lg[0], lg[1])
        assert nxt[1] == int(np.argmax(lp))


def cpu_threads():
    return len(os.sched_getaffinity(0))


@pytest.mark.parametrize("workload,layers,steps,n_ref", [
    ("llama3-8b-q8_0", 32, 3, 4),
    ("qwen2-72b-q4_1", 2, 3, 8),
])
def test_batch32_full_width_vs_reference(cuda, ref, workload, layers, steps, n_ref):
    """Batch 32 at the full 8B (32 layers) and 72B (2 layers, full width)
    shapes from seeded K/V states at depths up to 96: every sequence's greedy
    ids equal the single-token GPU step's (itself pinned to the reference at
    these shapes), and the first n_ref sequences equal the reference CPU path's
    independent contexts."""
    cfg, qtype, bias = C.WORKLOADS[workload]
    cfg = dict(cfg, n_layers=layers, max_seq_len=256)
    model = mlb.CudaModel(cfg).synthesize(qtype, SEED, with_bias=bias)
    n = 32
    rng = np.random.default_rng(1)
    depths = [int(d) for d in rng.integers(0, 96, n)]
    toks = [int(t) for t in rng.integers(0, cfg["vocab_size"], n)]
    b = mlb.Batch(model, n)
    for s in range(n):
        b.fill_kv(s, depths[s], 500 + s)
    got = b.decode_greedy(toks, depths, steps)
    ctx = model.context()
    for s in range(n):
        ctx.reset()
        ctx.fill_kv(depths[s], 500 + s)
        assert list(got[:, s]) == ctx.decode_greedy(toks[s], depths[s], steps), s
    ctx.close()
    b.close()
    r = ref
    r.set_threads(cpu_threads())
    rm = r.model(cfg).synthesize(qtype, SEED, bias, threads=cpu_threads())
    for s in range(n_ref):
        rm.new_context()  # a fresh MiniLlamaContext per sequence
        rm.fill_kv(depths[s], 500 + s)
        tok = toks[s]
        for i in range(steps):
            tok = int(np.argmax(rm.forward_token(tok, depths[s] + i)))
            assert tok == int(got[i, s]), (s, i)


def port_fill_kv(pm, n_pos, seed, scale=1.25, bf16=False):
    """The values mlb_batch_fill_kv writes (mlb_context_fill_kv's definition:
    generator streams 15 * 2^20 + l for K, 16 * 2^20 + l for V, element index
    (pos * KV + kv_head) * D + d, times scale), into the C port's cache,
    rounded to bf16 when the cache is bf16."""
    from mini_llama_b200 import _lib

    cfg = pm.cfg
    kd = cfg["n_kv_heads"] * cfg["head_dim"]
    keys, values = pm.kv_cache()
    s = _lib.synth_lib()
    for layer in range(cfg["n_layers"]):
        for kind, dst in ((15, keys), (16, values)):
            out = np.empty((n_pos, kd), np.float32)
            s.mlbs_f32(C.stream_key(seed, kind, layer), scale, 0, n_pos, 0, kd, kd,
                       out.ctypes.data, 4)
            if bf16:
                u = out.view(np.uint32).astype(np.uint64)
                u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
                out = u.astype(np.uint32).view(np.float32)
            dst[layer, :n_pos] = out.reshape(n_pos, cfg["n_kv_heads"], cfg["head_dim"])


@pytest.mark.parametrize("name", ["small_q4_0_gqa", "small_q4_1_neox_bias"])
def test_batch_bf16_kv_cache_matches_oracle(cuda, port, name):
    """A bf16 KV cache (mlb_batch_create_kv, MLB_KV_BF16): sequences at
    different depths decoded in lockstep against the C port with every K and V
    value rounded to bf16 when written (the seeded fill included): greedy ids
    equal, and one pass's logits within the bar."""
    mt = meta()[name]
    cfg = mt["config"]
    qtype = {v: k for k, v in C.QTYPE_NAMES.items()}[mt["qtype"]]
    model = mlb.CudaModel(cfg).synthesize(qtype, 17, with_bias=mt["bias"])
    n_seqs, steps = 4, 8
    depths = [0, 5, 11, 2]
    toks = [3, 77, 150, 9]
    b = mlb.Batch(model, n_seqs, kv_type=mlb.KV_BF16)
    for s in range(n_seqs):
        b.fill_kv(s, depths[s], 100 + s)
    got = b.decode_greedy(toks, depths, steps)
    for s in range(n_seqs):
        pm = port_model(port, cfg, qtype, 17, mt["bias"])
        pm.set_kv_bf16(True)
        port_fill_kv(pm, depths[s], 100 + s, bf16=True)
        tok = toks[s]
        for i in range(steps):
            tok = int(np.argmax(pm.forward_token(tok, depths[s] + i)))
            assert tok == int(got[i, s]), (s, i)
    # one pass with logits against the port
    b2 = mlb.Batch(model, 2, kv_type=mlb.KV_BF16)
    pm = port_model(port, cfg, qtype, 17, mt["bias"])
    pm.set_kv_bf16(True)
    for pos, t in enumerate([5, 6, 7, 8]):
        _, lg = b2.forward([0, 1], [t, t], [pos, pos], logits=True)
        lp = pm.forward_token(t, pos)
        assert np.abs(lg[0] - lp).max() <= LOGIT_TOL
        assert np.array_equal(lg[0], lg[1])


def _hd128(dim, heads, kv, max_seq, rope_type):
    return {"vocab_size": 512, "dim": dim, "hidden_dim": 512, "n_layers": 2, "n_heads": heads,
            "n_kv_heads": kv, "head_dim": 128, "max_seq_len": max_seq, "rope_theta": 1000000.0,
            "rms_norm_eps": 1e-06, "rope_type": rope_type}


# head_dim 128 with 8, 4 and 2 query heads per KV head: the bf16 cache's
# tensor-core attention kernel (smaller head_dim takes the register kernel)
HD128 = {
    "g8_q4_1_bias": (_hd128(1024, 8, 1, 1024, 1), C.Q4_1, True),
    "g4_q8_0": (_hd128(512, 4, 1, 512, 0), C.Q8_0, False),
    "g2_q4_0": (_hd128(512, 4, 2, 512, 0), C.Q4_0, False),
}


@pytest.mark.parametrize("name", list(HD128))
def test_batch_bf16_kv_head_dim_128(cuda, port, name):
    """Batched decode over a bf16 cache at head_dim 128 (tensor-core attention):
    sequences at ragged depths (empty and partial 16-position blocks, splits
    with no positions) against the C port with bf16-rounded K and V: greedy ids
    equal, one pass's logits within the bar."""
    cfg, qtype, bias = HD128[name]
    model = mlb.CudaModel(cfg).synthesize(qtype, 19, with_bias=bias)
    n_seqs, steps = 4, 6
    depths = [0, 37, 290, 130]
    toks = [3, 77, 150, 9]
    b = mlb.Batch(model, n_seqs, kv_type=mlb.KV_BF16)
    for s in range(n_seqs):
        b.fill_kv(s, depths[s], 200 + s)
    got = b.decode_greedy(toks, depths, steps)
    for s in range(n_seqs):
        pm = port_model(port, cfg, qtype, 19, bias)
        pm.set_kv_bf16(True)
        port_fill_kv(pm, depths[s], 200 + s, bf16=True)
        tok = toks[s]
        for i in range(steps):
            lp = pm.forward_token(tok, depths[s] + i)
            tok = int(np.argmax(lp))
            assert tok == int(got[i, s]), (s, i)
    b2 = mlb.Batch(model, 2, kv_type=mlb.KV_BF16)
    b2.fill_kv(0, 300, 9)
    b2.fill_kv(1, 300, 9)
    pm = port_model(port, cfg, qtype, 19, bias)
    pm.set_kv_bf16(True)
    port_fill_kv(pm, 300, 9, bf16=True)
    _, lg = b2.forward([0, 1], [5, 5], [300, 300], logits=True)
    lp = pm.forward_token(5, 300)
    assert np.abs(lg[0] - lp).max() <= LOGIT_TOL
    assert np.array_equal(lg[0], lg[1])


def test_batch_bf16_kv_head_dim_128_deep(cuda, port):
    """64 sequences at depth 3000 (G = 8, head_dim 128): 64 rows of one KV head
    make 19 splits of about 160 positions, so warps of the tensor-core
    attention kernel run two 16-position blocks (the online softmax's
    rescaling between blocks). Greedy ids and logits of three sequences
    against the port."""
    cfg, qtype, bias = HD128["g8_q4_1_bias"]
    cfg = dict(cfg, max_seq_len=4096)
    model = mlb.CudaModel(cfg).synthesize(qtype, 29, with_bias=bias)
    n_seqs, depth, steps = 64, 3000, 3
    b = mlb.Batch(model, n_seqs, kv_type=mlb.KV_BF16)
    for s in range(n_seqs):
        b.fill_kv(s, depth, 500 + s)
    toks = [(7 * s + 1) % cfg["vocab_size"] for s in range(n_seqs)]
    _, lg = b.forward(list(range(n_seqs)), toks, [depth] * n_seqs, logits=True)
    b.reset()
    for s in range(n_seqs):
        b.fill_kv(s, depth, 500 + s)
    got = b.decode_greedy(toks, [depth] * n_seqs, steps)
    for s in (0, 31, 63):
        pm = port_model(port, cfg, qtype, 29, bias)
        pm.set_kv_bf16(True)
        port_fill_kv(pm, depth, 500 + s, bf16=True)
        lp = pm.forward_token(toks[s], depth)
        assert np.abs(lg[s] - lp).max() <= LOGIT_TOL, s
        tok = int(np.argmax(lp))
        assert tok == int(got[0, s]), s
        for i in range(1, steps):
            tok = int(np.argmax(pm.forward_token(tok, depth + i)))
            assert tok == int(got[i, s]), (s, i)


def test_prefill_bf16_kv_head_dim_128(cuda, port):
    """A 300-token prompt through ForwardBatch into a bf16 context (G = 8,
    head_dim 128; passes of 64 rows at growing depths), then decoding on the
    step kernel: last-token logits and the decode against the port."""
    cfg, qtype, bias = HD128["g8_q4_1_bias"]
    model = mlb.CudaModel(cfg).synthesize(qtype, 23, with_bias=bias)
    pm = port_model(port, cfg, qtype, 23, bias)
    pm.set_kv_bf16(True)
    rng = np.random.default_rng(11)
    prompt = [int(t) for t in rng.integers(0, cfg["vocab_size"], 300)]
    for pos, t in enumerate(prompt):
        lp = pm.forward_token(t, pos)
    ctx = model.context(mlb.ATTN_CPU_COMPAT, kv_type=mlb.KV_BF16)
    lb = ctx.forward_batch(prompt, list(range(len(prompt))))
    assert np.abs(lb - lp).max() <= LOGIT_TOL
    tok = int(np.argmax(lp))
    assert int(np.argmax(lb)) == tok
    for pos in range(len(prompt), len(prompt) + 3):
        la, lc = ctx.forward_token(tok, pos), pm.forward_token(tok, pos)
        assert np.abs(la - lc).max() <= LOGIT_TOL, pos
        tok = int(np.argmax(lc))
    ctx.close()


def test_batch_kv_type_validation(cuda):
    cfg = meta()["small_q4_0_gqa"]["config"]
    model = mlb.CudaModel(cfg).synthesize(C.Q4_0, 3)
    with pytest.raises(mlb.MlbError, match="unknown KV cache type"):
        mlb.Batch(model, 2, kv_type=7)
