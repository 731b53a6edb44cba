"""GGUF v3 files of this package's models (seeded synthetic weights, or any
(kind, layer, qtype, rows, cols, array) list), for mlb_model_load_gguf, the
reference's LoadGgufModel and other GGUF readers.

Writes the published GGUF layout: magic "GGUF", version, tensor and metadata
counts, metadata key/value pairs, tensor infos (name, dims with the row length
first, ggml type, offset into the data section), padding to the alignment,
then the tensor data, each tensor at an aligned offset. The metadata keys are
the ones the reference's BuildConfig reads (src/gguf_loader.cc:13-88) and the
tensor names the ones MapTensorName maps (src/gguf_loader.cc:91-160).
"""
from __future__ import annotations

import struct

import numpy as np

from . import configs as C

# ggml tensor types
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_1, GGML_Q8_0 = 0, 1, 2, 3, 8
GGML_OF_QTYPE = {C.F32: GGML_F32, C.Q8_0: GGML_Q8_0, C.Q4_0: GGML_Q4_0, C.Q4_1: GGML_Q4_1}

# metadata value types
U32, I32, F32V, STR, ARR, U64 = 4, 5, 6, 8, 9, 10

LAYER_NAMES = {
    C.W_ATTENTION_NORM: "attn_norm.weight", C.W_WQ: "attn_q.weight", C.W_WK: "attn_k.weight",
    C.W_WV: "attn_v.weight", C.W_BQ: "attn_q.bias", C.W_BK: "attn_k.bias",
    C.W_BV: "attn_v.bias", C.W_WO: "attn_output.weight", C.W_FFN_NORM: "ffn_norm.weight",
    C.W_GATE: "ffn_gate.weight", C.W_UP: "ffn_up.weight", C.W_DOWN: "ffn_down.weight",
}
GLOBAL_NAMES = {C.W_TOKEN_EMBEDDING: "token_embd.weight", C.W_FINAL_NORM: "output_norm.weight",
                C.W_LM_HEAD: "output.weight"}


def tensor_name(kind: int, layer: int) -> str:
    if kind in GLOBAL_NAMES:
        return GLOBAL_NAMES[kind]
    return f"blk.{layer}.{LAYER_NAMES[kind]}"


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v) -> bytes:
    if vtype == U32:
        return struct.pack("<I", v)
    if vtype == I32:
        return struct.pack("<i", v)
    if vtype == U64:
        return struct.pack("<Q", v)
    if vtype == F32V:
        return struct.pack("<f", v)
    if vtype == STR:
        return _str(v)
    if vtype == ARR:
        etype, items = v
        return struct.pack("<IQ", etype, len(items)) + b"".join(_value(etype, x) for x in items)
    raise ValueError(vtype)


def model_metadata(cfg: dict, arch: str | None = None, alignment: int | None = None):
    """(key, type, value) list for a model config."""
    arch = arch or ("qwen2" if cfg.get("rope_type", 0) == 1 else "llama")
    meta = [
        ("general.architecture", STR, arch),
        (f"{arch}.block_count", U32, cfg["n_layers"]),
        (f"{arch}.embedding_length", U32, cfg["dim"]),
        (f"{arch}.feed_forward_length", U32, cfg["hidden_dim"]),
        (f"{arch}.attention.head_count", U32, cfg["n_heads"]),
        (f"{arch}.attention.head_count_kv", U32, cfg["n_kv_heads"]),
        (f"{arch}.context_length", U32, cfg["max_seq_len"]),
        (f"{arch}.rope.freq_base", F32V, float(cfg["rope_theta"])),
        (f"{arch}.attention.layer_norm_rms_epsilon", F32V, float(cfg["rms_norm_eps"])),
        ("tokenizer.ggml.tokens", ARR, (STR, [f"<t{i}>" for i in range(cfg["vocab_size"])])),
    ]
    if alignment is not None:
        meta.append(("general.alignment", U32, alignment))
    return meta


def data_bytes(gtype: int, dims) -> int:
    n = 1
    for d in dims:
        n *= d
    if gtype == GGML_F32:
        return 4 * n
    if gtype == GGML_F16:
        return 2 * n
    return (n + 31) // 32 * {GGML_Q4_0: 18, GGML_Q4_1: 20, GGML_Q8_0: 34}[gtype]


def write_gguf(path: str, meta, tensors, alignment: int = 32, version: int = 3,
               magic: bytes = b"GGUF") -> None:
    """tensors: (name, ggml_type, dims with the row length first, data), data
    bytes / an array, or a callable returning them (called once, in order, so
    a large model is generated one tensor at a time)."""
    head = bytearray(magic + struct.pack("<IQQ", version, len(tensors), len(meta)))
    for key, vtype, v in meta:
        head += _str(key) + struct.pack("<I", vtype) + _value(vtype, v)
    offsets, sizes, off = [], [], 0
    for name, gtype, dims, data in tensors:
        n = len(data) if isinstance(data, (bytes, bytearray)) else data_bytes(gtype, dims)
        offsets.append(off)
        sizes.append(n)
        off = (off + n + alignment - 1) // alignment * alignment
    for (name, gtype, dims, data), o in zip(tensors, offsets):
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", gtype, o)
    pad = (-len(head)) % alignment
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        pos = 0
        for (name, gtype, dims, data), o, n in zip(tensors, offsets, sizes):
            if callable(data):
                data = data()
            buf = memoryview(np.ascontiguousarray(data)).cast("B") if not isinstance(
                data, (bytes, bytearray)) else data
            if len(buf) != n:
                raise ValueError(f"{name}: {len(buf)} bytes, expected {n}")
            f.write(b"\0" * (o - pos))
            f.write(buf)
            pos = o + n


def model_tensors(weights, f16_linear: bool = False, drop=()):
    """GGUF tensors from (kind, layer, qtype, rows, cols, array) weights.
    f16_linear: F32 linear weights are stored as F16. drop: kinds left out."""
    out = []
    for kind, layer, qtype, rows, cols, arr in weights:
        if kind in drop:
            continue
        one_d = rows == 1 and kind not in (C.W_TOKEN_EMBEDDING, C.W_LM_HEAD)
        dims = [cols] if one_d else [cols, rows]
        linear = kind in (C.W_WQ, C.W_WK, C.W_WV, C.W_WO, C.W_GATE, C.W_UP, C.W_DOWN, C.W_LM_HEAD)
        if qtype == C.F32 and f16_linear and linear:
            data = np.ascontiguousarray(arr, np.float32).astype(np.float16).tobytes()
            gtype = GGML_F16
        else:
            data = np.ascontiguousarray(arr).tobytes()
            gtype = GGML_OF_QTYPE[qtype]
        out.append((tensor_name(kind, layer), gtype, dims, data))
    return out


def write_synthetic_model(path: str, cfg: dict, qtype: int, seed: int, with_bias: bool = False,
                          threads: int = 8) -> int:
    """The seeded model CudaModel.synthesize builds (the bytes of
    configs.host_weights), written as GGUF one tensor at a time. Returns the
    file size."""
    import os

    entries = []
    for layer in range(cfg["n_layers"]):
        for kind in C.LAYER_KINDS:
            if kind in (C.W_BQ, C.W_BK, C.W_BV) and not with_bias:
                continue
            entries.append((kind, layer))
    entries += [(C.W_TOKEN_EMBEDDING, -1), (C.W_FINAL_NORM, -1), (C.W_LM_HEAD, -1)]
    tensors = []
    for kind, layer in entries:
        rows, cols = C.weight_shape(cfg, kind)
        if kind in (C.W_ATTENTION_NORM, C.W_FFN_NORM, C.W_FINAL_NORM):
            qt, fn = C.F32, (lambda r=rows, c=cols: np.ones((r, c), np.float32))
        elif kind in (C.W_BQ, C.W_BK, C.W_BV, C.W_TOKEN_EMBEDDING):
            qt = C.F32
            fn = (lambda k=kind, l=layer, r=rows, c=cols:
                  C.synth_tensor(seed, k, l, C.F32, r, c, threads))
        else:
            qt = qtype
            fn = (lambda k=kind, l=layer, r=rows, c=cols:
                  C.synth_tensor(seed, k, l, qtype, r, c, threads))
        one_d = rows == 1 and kind not in (C.W_TOKEN_EMBEDDING, C.W_LM_HEAD)
        tensors.append((tensor_name(kind, layer), GGML_OF_QTYPE[qt], [cols] if one_d else [cols, rows],
                        fn))
    write_gguf(path, model_metadata(cfg), tensors)
    return os.path.getsize(path)
