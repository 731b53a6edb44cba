"""The bf16 KV cache of a single context (mlb_context_create_kv, MLB_KV_BF16):
the decode step kernel writes K and V rounded to bf16 (nearest even) and its
attention phase widens them exactly. Not a reference mode (the reference's
CudaKvCache is fp32, src/cuda_kv_cache.cc:60-92); the comparator is the C port
with the same switch (every K and V value rounded to bf16 when written), on
the golden small models (GQA, NeoX + q/k/v bias, ragged shapes):

* greedy ids bit-exact and logits within 2e-3 per step, from position 0 and
  from a seeded K/V state;
* ForwardBatch (prompt prefill through the batched engine) into a bf16
  context continues the decode like the port;
* the option is refused where it cannot run (the per-op path).
"""
import json

import numpy as np
import pytest

import mini_llama_b200 as mlb
from mini_llama_b200 import configs as C
from tests.conftest import golden_path
from tests.test_gpu_batch import port_fill_kv, port_model

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3
NAMES = ["small_q4_0_gqa", "small_q4_1_neox_bias", "small_q8_0_ragged"]


def small(name):
    with open(golden_path("golden.json")) as f:
        mt = json.load(f)[name]
    qtype = {v: k for k, v in C.QTYPE_NAMES.items()}[mt["qtype"]]
    return mt["config"], qtype, mt["bias"]


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("depth", [0, 9])
def test_step_kernel_bf16_kv_matches_port(cuda, port, name, depth):
    cfg, qtype, bias = small(name)
    model = mlb.CudaModel(cfg).synthesize(qtype, 41, with_bias=bias)
    ctx = model.context(mlb.ATTN_CPU_COMPAT, kv_type=mlb.KV_BF16)
    assert ctx.step_kernel()
    pm = port_model(port, cfg, qtype, 41, bias)
    pm.set_kv_bf16(True)
    if depth:
        ctx.fill_kv(depth, 300)
        port_fill_kv(pm, depth, 300, bf16=True)
    tok = 11
    for pos in range(depth, depth + 8):
        lg = ctx.forward_token(tok, pos)
        lp = pm.forward_token(tok, pos)
        assert np.abs(lg - lp).max() <= LOGIT_TOL, pos
        assert int(np.argmax(lg)) == int(np.argmax(lp)), pos
        tok = int(np.argmax(lp))
    # the on-device greedy loop decodes the same ids
    ctx.reset()
    pm2 = port_model(port, cfg, qtype, 41, bias)
    pm2.set_kv_bf16(True)
    if depth:
        ctx.fill_kv(depth, 300)
        port_fill_kv(pm2, depth, 300, bf16=True)
    want, t = [], 11
    for pos in range(depth, depth + 6):
        t = int(np.argmax(pm2.forward_token(t, pos)))
        want.append(t)
    assert ctx.decode_greedy(11, depth, 6) == want
    ctx.close()


def test_forward_batch_into_bf16_context(cuda, port):
    cfg, qtype, bias = small("small_q4_1_neox_bias")
    model = mlb.CudaModel(cfg).synthesize(qtype, 43, with_bias=bias)
    pm = port_model(port, cfg, qtype, 43, bias)
    pm.set_kv_bf16(True)
    rng = np.random.default_rng(4)
    prompt = [int(t) for t in rng.integers(0, cfg["vocab_size"], 20)]
    for pos, t in enumerate(prompt):
        lp = pm.forward_token(t, pos)
    ctx = model.context(mlb.ATTN_CPU_COMPAT, kv_type=mlb.KV_BF16)
    lb = ctx.forward_batch(prompt, list(range(len(prompt))))
    assert np.abs(lb - lp).max() <= LOGIT_TOL
    tok = int(np.argmax(lp))
    for pos in range(len(prompt), len(prompt) + 4):
        la, lc = ctx.forward_token(tok, pos), pm.forward_token(tok, pos)
        assert np.abs(la - lc).max() <= LOGIT_TOL, pos
        tok = int(np.argmax(lc))
    ctx.close()


def test_bf16_kv_refusals(cuda):
    cfg, qtype, bias = small("small_q4_0_gqa")
    model = mlb.CudaModel(cfg).synthesize(qtype, 3)
    ctx = model.context(kv_type=mlb.KV_BF16)
    with pytest.raises(mlb.MlbError, match="step kernel only"):
        ctx.set_step_kernel(False)
    ctx.close()
    with pytest.raises(mlb.MlbError, match="unknown KV cache type"):
        model.context(kv_type=5)
    # F32 weights: the step kernel does not take the model, so neither does bf16
    f32 = mlb.CudaModel(cfg).load(C.host_weights(cfg, C.F32, 3))
    with pytest.raises(mlb.MlbError, match="needs the decode step kernel"):
        f32.context(kv_type=mlb.KV_BF16)
