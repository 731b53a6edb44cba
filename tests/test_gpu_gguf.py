"""GGUF files loaded onto the GPU (mlb_model_load_gguf, csrc/gguf.cu) against
the reference's own LoadGgufModel (src/gguf_loader.cc:302-418) reading the
same file on the CPU (oracle/_ref).

* quantised models (Q4_0 GQA, Q4_1 NeoX with q/k/v bias, Q8_0 ragged): greedy
  ids equal to the reference's, logits within 2e-3 per step, and bit-equal to
  the same weights uploaded through mlb_model_set_weight;
* an embedding stored as Q8_0 and no output.weight (tied lm_head): both
  loaders dequantise the embedding and tie the lm_head to it;
* F16 linear weights, which the reference rejects: compared with the
  reference reading the same values widened to F32 (exact).
"""
import json

import numpy as np
import pytest

import mini_llama_b200 as mlb
from mini_llama_b200 import configs as C
from mini_llama_b200 import gguf_writer as GW
from tests.conftest import golden_path

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3


def small(name):
    with open(golden_path("golden.json")) as f:
        mt = json.load(f)[name]
    qtype = {v: k for k, v in C.QTYPE_NAMES.items()}[mt["qtype"]]
    return mt["config"], qtype, mt["bias"]


def decode_both(gpu_model, ref_model, steps=8, tok=7):
    ctx = gpu_model.context(mlb.ATTN_CPU_COMPAT)
    out = []
    for pos in range(steps):
        lg = ctx.forward_token(tok, pos)
        lr = ref_model.forward_token(tok, pos)
        assert np.abs(lg - lr).max() <= LOGIT_TOL, pos
        assert int(np.argmax(lg)) == int(np.argmax(lr)), pos
        out.append(lg)
        tok = int(np.argmax(lr))
    ctx.close()
    return out


@pytest.mark.parametrize("name", ["small_q4_0_gqa", "small_q4_1_neox_bias", "small_q8_0_ragged"])
def test_load_gguf_matches_reference_loader(cuda, ref, tmp_path, name):
    cfg, qtype, bias = small(name)
    weights = list(C.host_weights(cfg, qtype, 21, bias))
    p = tmp_path / "m.gguf"
    GW.write_gguf(str(p), GW.model_metadata(cfg), GW.model_tensors(weights))
    gm = mlb.CudaModel.from_gguf(str(p))
    assert gm.gguf_bytes > 0
    got = decode_both(gm, ref.load_gguf(str(p)))
    # the same weights through mlb_model_set_weight: the same device model
    sm = mlb.CudaModel(cfg).load(weights)
    ctx = sm.context(mlb.ATTN_CPU_COMPAT)
    tok = 7
    for pos, lg in enumerate(got):
        ls = ctx.forward_token(tok, pos)
        assert np.array_equal(ls, lg), pos
        tok = int(np.argmax(lg))
    ctx.close()


def test_quantised_embedding_and_tied_lm_head(cuda, ref, tmp_path):
    cfg, qtype, bias = small("small_q4_0_gqa")
    weights = list(C.host_weights(cfg, qtype, 23, bias))
    emb = next(w for w in weights if w[0] == C.W_TOKEN_EMBEDDING)
    q = ref.quantize(C.Q8_0, emb[5])  # the reference's own QuantizeToQ80
    tensors = []
    for t in GW.model_tensors(weights, drop=(C.W_LM_HEAD,)):
        if t[0] == "token_embd.weight":
            t = (t[0], GW.GGML_Q8_0, t[2], np.ascontiguousarray(q).tobytes())
        tensors.append(t)
    p = tmp_path / "tied.gguf"
    GW.write_gguf(str(p), GW.model_metadata(cfg), tensors)
    decode_both(mlb.CudaModel.from_gguf(str(p)), ref.load_gguf(str(p)))


def test_f16_linear_weights(cuda, ref, tmp_path):
    """F16 linear weights load (widened to F32); the reference, which rejects
    F16, reads the same values stored as F32."""
    cfg, _, _ = small("small_q4_0_gqa")
    weights = list(C.host_weights(cfg, C.F32, 29, False))
    widened = []
    for kind, layer, qt, rows, cols, arr in weights:
        if kind in (C.W_WQ, C.W_WK, C.W_WV, C.W_WO, C.W_GATE, C.W_UP, C.W_DOWN, C.W_LM_HEAD):
            arr = np.asarray(arr, np.float32).astype(np.float16).astype(np.float32)
        widened.append((kind, layer, qt, rows, cols, arr))
    p16, p32 = tmp_path / "f16.gguf", tmp_path / "f32.gguf"
    GW.write_gguf(str(p16), GW.model_metadata(cfg), GW.model_tensors(widened, f16_linear=True))
    GW.write_gguf(str(p32), GW.model_metadata(cfg), GW.model_tensors(widened))
    with pytest.raises(RuntimeError, match="Unsupported GGUF tensor type: 1"):
        ref.load_gguf(str(p16))
    decode_both(mlb.CudaModel.from_gguf(str(p16)), ref.load_gguf(str(p32)))


def test_load_gguf_errors(cuda, tmp_path):
    cfg, qtype, bias = small("small_q4_0_gqa")
    weights = list(C.host_weights(cfg, qtype, 3, bias))
    p = tmp_path / "missing.gguf"
    GW.write_gguf(str(p), GW.model_metadata(cfg),
                  [t for t in GW.model_tensors(weights) if t[0] != "blk.1.ffn_down.weight"])
    with pytest.raises(mlb.MlbError, match="Missing tensor: layers.1.w_down"):
        mlb.CudaModel.from_gguf(str(p))
    bad = dict(cfg, hidden_dim=cfg["hidden_dim"] + 32)
    p = tmp_path / "shape.gguf"
    GW.write_gguf(str(p), GW.model_metadata(bad), GW.model_tensors(weights))
    with pytest.raises(mlb.MlbError, match="shape mismatch"):
        mlb.CudaModel.from_gguf(str(p))
