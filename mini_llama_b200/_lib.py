"""ctypes binding of include/mlb200.h (libmlb200.so) and libmlb_synth.so.

The CUDA library is required: loading fails loudly when it is missing and
cannot be built; there is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes
import os

from . import build as _build

HERE = os.path.dirname(os.path.abspath(__file__))

_c_int, _c_size_t, _c_float, _c_u64 = ctypes.c_int, ctypes.c_size_t, ctypes.c_float, ctypes.c_uint64
_vp, _fp = ctypes.c_void_p, ctypes.POINTER(ctypes.c_float)
_ip = ctypes.POINTER(ctypes.c_int)


class MlbConfig(ctypes.Structure):
    """mlb_config, mirroring ModelConfig (include/mini_llama/model.h:21-33)."""

    _fields_ = [(n, ctypes.c_int) for n in ("vocab_size", "dim", "hidden_dim", "n_layers",
                                             "n_heads", "n_kv_heads", "head_dim",
                                             "max_seq_len")] + [
        ("rope_theta", ctypes.c_float), ("rms_norm_eps", ctypes.c_float),
        ("rope_type", ctypes.c_int)]


class MlbTpShard(ctypes.Structure):
    """mlb_tp_shard: the rows / input columns one tensor-parallel rank keeps."""

    _fields_ = [(n, ctypes.c_int) for n in ("q_head0", "q_heads", "kv_head0", "kv_heads",
                                             "ffn_row0", "ffn_rows", "vocab_row0",
                                             "vocab_rows")]


# (name, restype, argtypes) of every entry point in include/mlb200.h
SIGNATURES = [
    ("mlb_last_error", ctypes.c_char_p, []),
    ("mlb_built", _c_int, []),
    ("mlb_device_count", _c_int, [_ip]),
    ("mlb_wait_selftest", _c_int, [_c_int, _c_int, ctypes.c_double, _ip, _ip]),
    ("mlb_linear", _c_int, [_c_int, _vp, _c_int, _c_int, _vp, _c_size_t, _c_int, _vp, _c_int, _vp]),
    ("mlb_linear_host", _c_int, [_c_int, _vp, _c_int, _c_int, _vp, _c_size_t, _c_int, _vp, _vp,
                                 _c_int]),
    ("mlb_linear_device_weight", _c_int, [_c_int, _vp, _c_int, _c_int, _vp, _c_size_t, _c_int,
                                          _vp, _vp, _c_int]),
    ("mlb_rmsnorm", _c_int, [_vp, _vp, _c_int, _c_float, _vp, _c_int, _vp]),
    ("mlb_silu", _c_int, [_vp, _c_int, _vp, _c_int, _vp]),
    ("mlb_mul", _c_int, [_vp, _vp, _c_int, _vp, _c_int, _vp]),
    ("mlb_add", _c_int, [_vp, _vp, _c_int, _vp, _c_int, _vp]),
    ("mlb_softmax", _c_int, [_vp, _c_int, _vp, _c_int, _vp]),
    ("mlb_embedding", _c_int, [_vp, _c_int, _c_int, _c_int, _vp, _c_int, _vp]),
    ("mlb_rope", _c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_float, _c_int, _c_int, _vp]),
    ("mlb_argmax", _c_int, [_vp, _c_int, _ip, _c_int, _vp]),
    ("mlb_kv_write", _c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _vp,
                              _c_int, _vp]),
    ("mlb_attention_decode", _c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                      _c_int, _c_int, _c_int, _vp, _c_int, _vp]),
    ("mlb_attention_decode_noalloc", _c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                              _c_int, _c_int, _c_int, _c_int, _vp, _c_int, _vp]),
    ("mlb_qmatrix_create", _c_int, [_c_int, _vp, _c_int, _c_int, _c_int, _c_int,
                                    ctypes.POINTER(_vp)]),
    ("mlb_qmatrix_synthesize", _c_int, [_c_int, _c_int, _c_int, _c_u64, _c_u64, _c_int, _c_int,
                                        ctypes.POINTER(_vp)]),
    ("mlb_qmatrix_gemv", _c_int, [_vp, _vp, _c_int, _vp, _vp]),
    ("mlb_qmatrix_gemm", _c_int, [_vp, _vp, _c_int, _vp, _vp]),
    ("mlb_qmatrix_dequant", _c_int, [_vp, _vp, _vp]),
    ("mlb_qmatrix_bytes", _c_size_t, [_vp]),
    ("mlb_qmatrix_destroy", _c_int, [_vp]),
    ("mlb_tp_plan", _c_int, [ctypes.POINTER(MlbConfig), _c_int, _c_int,
                             ctypes.POINTER(MlbTpShard)]),
    ("mlb_model_create", _c_int, [ctypes.POINTER(MlbConfig), _c_int, _c_int, _c_int, _vp,
                                  ctypes.POINTER(_vp)]),
    ("mlb_model_set_weight", _c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _c_size_t]),
    ("mlb_model_synthesize", _c_int, [_vp, _c_int, _c_u64, _c_int]),
    ("mlb_model_finalize", _c_int, [_vp]),
    ("mlb_model_destroy", _c_int, [_vp]),
    ("mlb_model_bytes", _c_int, [_vp, ctypes.POINTER(_c_size_t), ctypes.POINTER(_c_size_t)]),
    ("mlb_gguf_read_config", _c_int, [ctypes.c_char_p, ctypes.POINTER(MlbConfig)]),
    ("mlb_model_load_gguf", _c_int, [ctypes.c_char_p, _c_int, _c_int, _c_int, _vp, _c_int,
                                     ctypes.POINTER(_vp), ctypes.POINTER(_c_size_t)]),
    ("mlb_context_create", _c_int, [_vp, _c_int, ctypes.POINTER(_vp)]),
    ("mlb_context_create_kv", _c_int, [_vp, _c_int, _c_int, ctypes.POINTER(_vp)]),
    ("mlb_context_destroy", _c_int, [_vp]),
    ("mlb_context_reset", _c_int, [_vp]),
    ("mlb_context_fill_kv", _c_int, [_vp, _c_int, _c_u64, _c_float]),
    ("mlb_forward_token", _c_int, [_vp, _c_int, _c_int, _vp]),
    ("mlb_forward_token_device", _c_int, [_vp, _c_int, _c_int, ctypes.POINTER(_vp)]),
    ("mlb_context_sync", _c_int, [_vp]),
    ("mlb_decode_greedy", _c_int, [_vp, _c_int, _c_int, _c_int, _vp]),
    ("mlb_context_stream", _vp, [_vp]),
    ("mlb_context_kernels_per_step", _c_int, [_vp]),
    ("mlb_context_set_step_kernel", _c_int, [_vp, _c_int]),
    ("mlb_context_step_kernel", _c_int, [_vp]),
    ("mlb_context_step_trace", _c_int, [_vp, _c_int]),
    ("mlb_context_step_trace_read", _c_int,
     [_vp, _vp, _c_size_t, ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]),
    ("mlb_nccl_unique_id", _c_int, [_vp]),
    ("mlb_sampler_create", _c_int, [_c_int, ctypes.c_uint, ctypes.POINTER(_vp)]),
    ("mlb_sampler_destroy", _c_int, [_vp]),
    ("mlb_sample", _c_int, [_vp, _vp, _c_int, _c_float, _c_int, ctypes.POINTER(_c_int)]),
    ("mlb_decode_sample", _c_int, [_vp, _vp, _c_float, _c_int, _c_int, _c_int, _c_int, _vp]),
    ("mlb_forward_batch", _c_int, [_vp, _c_int, _vp, _vp, _vp]),
    ("mlb_batch_create", _c_int, [_vp, _c_int, _c_int, ctypes.POINTER(_vp)]),
    ("mlb_batch_create_kv", _c_int, [_vp, _c_int, _c_int, _c_int, ctypes.POINTER(_vp)]),
    ("mlb_batch_destroy", _c_int, [_vp]),
    ("mlb_batch_reset", _c_int, [_vp]),
    ("mlb_batch_fill_kv", _c_int, [_vp, _c_int, _c_int, _c_u64, _c_float]),
    ("mlb_batch_forward", _c_int, [_vp, _c_int, _vp, _vp, _vp, _vp, _vp]),
    ("mlb_batch_decode_greedy", _c_int, [_vp, _vp, _vp, _c_int, _vp]),
    ("mlb_batch_stream", _vp, [_vp]),
    ("mlb_batch_kernels_per_step", _c_int, [_vp]),
]

SYNTH_SIGNATURES = [
    ("mlbs_stream_key", _c_u64, [_c_u64, _c_u64]),
    ("mlbs_stream_id", _c_u64, [_c_int, _c_int]),
    ("mlbs_gguf", None, [_c_int, _c_u64, _c_float, _c_int, ctypes.c_longlong, ctypes.c_longlong,
                         ctypes.c_longlong, ctypes.c_longlong, ctypes.c_longlong, _vp, _c_size_t,
                         _c_int]),
    ("mlbs_f32", None, [_c_u64, _c_float, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_longlong,
                        ctypes.c_longlong, ctypes.c_longlong, _vp, _c_int]),
    ("mlbs_quantize_block", None, [_c_int, _vp, _c_int, _vp]),
    ("mlbs_f32_to_fp16", ctypes.c_uint16, [_c_float]),
]

_lib = None
_synth = None


class MlbError(RuntimeError):
    """A failed call (the reference's std::runtime_error)."""

    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


class MlbRangeError(IndexError):
    """MLB_ERR_RANGE: the reference's std::out_of_range."""

    code = -2


def _bind(lib, sigs):
    for name, res, args in sigs:
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args


def lib():
    """The CUDA library; built in-tree on first use if absent."""
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "libmlb200.so")
        if not os.path.exists(path):
            _build.build_cuda()
        if not os.path.exists(path):
            raise RuntimeError("libmlb200.so is missing and could not be built")
        _lib = ctypes.CDLL(path)
        _bind(_lib, SIGNATURES)
    return _lib


def synth_lib():
    global _synth
    if _synth is None:
        path = os.path.join(HERE, "libmlb_synth.so")
        if not os.path.exists(path):
            _build.build_synth()
        _synth = ctypes.CDLL(path)
        _bind(_synth, SYNTH_SIGNATURES)
    return _synth


def check(rc: int) -> int:
    if rc != 0:
        msg = lib().mlb_last_error().decode(errors="replace")
        if rc == -2:
            raise MlbRangeError(msg)
        raise MlbError(rc, msg)
    return rc
