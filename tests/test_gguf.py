"""GGUF model files, host side: the config and parse behaviour of
mlb_gguf_read_config (csrc/gguf.cu) against the reference's own
LoadGgufModel (src/gguf_loader.cc:302-418, built into oracle/_ref), and the
package's writer (mini_llama_b200/gguf_writer.py) pinned by the reference reading its files
back into the same logits as the model built from the same weights.
No device is needed."""
import json
import struct

import numpy as np
import pytest

import mini_llama_b200 as mlb
from mini_llama_b200 import configs as C
from mini_llama_b200 import gguf_writer as GW
from tests.conftest import golden_path

SMALL = ["small_q4_0_gqa", "small_q4_1_neox_bias", "small_q8_0_ragged"]


def small(name):
    with open(golden_path("golden.json")) as f:
        mt = json.load(f)[name]
    qtype = {v: k for k, v in C.QTYPE_NAMES.items()}[mt["qtype"]]
    return mt["config"], qtype, mt["bias"]


def write_model(path, cfg, weights, **kw):
    GW.write_gguf(str(path), GW.model_metadata(cfg), GW.model_tensors(weights, **kw))


@pytest.mark.parametrize("name", SMALL)
def test_config_matches_reference_loader(ref, tmp_path, name):
    cfg, qtype, bias = small(name)
    p = tmp_path / "m.gguf"
    write_model(p, cfg, list(C.host_weights(cfg, qtype, 5, bias)))
    got = mlb.read_gguf_config(str(p))
    for k in ("vocab_size", "dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "head_dim",
              "max_seq_len", "rope_type"):
        assert got[k] == cfg[k], k
    assert got["rope_theta"] == np.float32(cfg["rope_theta"])
    assert got["rms_norm_eps"] == np.float32(cfg["rms_norm_eps"])
    rm = ref.load_gguf(str(p))
    for k in ("vocab_size", "dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "head_dim",
              "max_seq_len", "rope_type"):
        assert rm.cfg[k] == got[k], k


@pytest.mark.parametrize("name", ["small_q4_1_neox_bias", "small_q8_0_ragged"])
def test_reference_reads_writer_files(ref, tmp_path, name):
    """The writer is pinned: the reference's LoadGgufModel on its file decodes
    exactly the logits of the reference model given the same weights directly."""
    cfg, qtype, bias = small(name)
    weights = list(C.host_weights(cfg, qtype, 9, bias))
    p = tmp_path / "m.gguf"
    write_model(p, cfg, weights)
    a = ref.load_gguf(str(p))
    b = ref.model(cfg)
    for kind, layer, qt, rows, cols, arr in weights:
        b.set_weight(kind, layer, qt, rows, cols, arr)
    tok = 3
    for pos in range(4):
        la, lb = a.forward_token(tok, pos), b.forward_token(tok, pos)
        assert np.array_equal(la, lb), pos
        tok = int(np.argmax(la))


def _bytes_with(p, tmp_path, edit):
    raw = bytearray(p.read_bytes())
    edit(raw)
    q = tmp_path / "edited.gguf"
    q.write_bytes(bytes(raw))
    return str(q)


def test_parse_errors_match_reference(ref, tmp_path):
    cfg, qtype, bias = small("small_q4_0_gqa")
    p = tmp_path / "m.gguf"
    write_model(p, cfg, list(C.host_weights(cfg, qtype, 1, bias)))
    cases = {
        "invalid GGUF magic": lambda r: r.__setitem__(slice(0, 4), b"GGUX"),
        "unsupported GGUF version: 2": lambda r: r.__setitem__(slice(4, 8), struct.pack("<I", 2)),
    }
    for msg, edit in cases.items():
        q = _bytes_with(p, tmp_path, edit)
        with pytest.raises(mlb.MlbError, match=msg):
            mlb.read_gguf_config(q)
        with pytest.raises(RuntimeError, match=msg):
            ref.load_gguf(q)
    # a truncated file (tensor data cut off)
    q = tmp_path / "cut.gguf"
    q.write_bytes(p.read_bytes()[: p.stat().st_size // 2])
    with pytest.raises(mlb.MlbError, match="GGUF parse error"):
        mlb.read_gguf_config(str(q))
    with pytest.raises(RuntimeError, match="GGUF parse error"):
        ref.load_gguf(str(q))


def test_duplicate_metadata_key(tmp_path):
    cfg, _, _ = small("small_q4_0_gqa")
    meta = GW.model_metadata(cfg) + [("general.architecture", GW.STR, "llama")]
    p = tmp_path / "dup.gguf"
    GW.write_gguf(str(p), meta, [])
    with pytest.raises(mlb.MlbError, match="duplicate metadata key: general.architecture"):
        mlb.read_gguf_config(str(p))


def test_config_errors(tmp_path):
    cfg, _, _ = small("small_q4_0_gqa")
    meta = [m for m in GW.model_metadata(cfg) if not m[0].endswith("block_count")]
    p = tmp_path / "nolayers.gguf"
    GW.write_gguf(str(p), meta, [])
    with pytest.raises(mlb.MlbError, match="Invalid model config from GGUF: dim=256 layers=0"):
        mlb.read_gguf_config(str(p))
    # the qwen2.* keys win over llama.* ones, and qwen2 selects NeoX RoPE
    meta = GW.model_metadata(cfg, arch="llama") + [
        ("qwen2.block_count", GW.U32, 5)] + [("general.alignment", GW.U32, 64)]
    p = tmp_path / "mixed.gguf"
    GW.write_gguf(str(p), meta, [], alignment=64)
    got = mlb.read_gguf_config(str(p))
    assert got["n_layers"] == 5 and got["rope_type"] == 0


def test_bad_alignment(tmp_path):
    cfg, _, _ = small("small_q4_0_gqa")
    p = tmp_path / "align.gguf"
    GW.write_gguf(str(p), GW.model_metadata(cfg, alignment=48), [], alignment=48)
    with pytest.raises(mlb.MlbError, match="invalid general.alignment"):
        mlb.read_gguf_config(str(p))
