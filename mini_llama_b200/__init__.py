"""mini_llama_b200 — B200 (sm_100a) decode forward path of mini-llama.

Python mirror of the reference's device-branch interface, over the C ABI of
include/mlb200.h (libmlb200.so). Names follow the reference
(include/mini_llama/cuda_quant.h, cuda_matmul.h, cuda_ops.h, cuda_attention.h,
cuda_kv_cache.h, forward.h); device memory is held in torch CUDA tensors,
which here are plumbing only -- every computation runs in this package's own
kernels. Errors raise ``MlbError`` (the reference's std::runtime_error) or
``MlbRangeError`` (std::out_of_range) with the reference's messages.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import configs
from ._lib import MlbConfig, MlbError, MlbRangeError, check, lib, synth_lib
from .configs import (F32, Q4_0, Q4_1, Q8_0, W_BK, W_BQ, W_BV, W_DOWN, W_FFN_NORM,
                      W_FINAL_NORM, W_GATE, W_LM_HEAD, W_TOKEN_EMBEDDING, W_UP, W_WK, W_WO,
                      W_WQ, W_WV, W_ATTENTION_NORM)

ROPE_NORMAL, ROPE_NEOX = 0, 1
ATTN_CPU_COMPAT, ATTN_STANDARD = 0, 1
KV_F32, KV_BF16 = 0, 1  # MLB_KV_F32, MLB_KV_BF16: KV cache element type of a Batch
ERR_TIMEOUT = -5  # MLB_ERR_TIMEOUT: a bounded device wait gave up

__all__ = [
    "F32", "Q8_0", "Q4_0", "Q4_1", "ROPE_NORMAL", "ROPE_NEOX", "ATTN_CPU_COMPAT",
    "ATTN_STANDARD", "Sampler", "MlbError", "MlbRangeError", "CudaQuantBuilt", "CudaDeviceCount",
    "CudaQ80LinearDeviceInput", "CudaQ40LinearDeviceInput", "CudaQ41LinearDeviceInput",
    "CudaLinearDeviceInput", "CudaQ80Linear", "CudaQ40Linear", "CudaQ41Linear", "CudaLinear",
    "CudaRmsNormDeviceWeight", "CudaSiluDeviceInput", "CudaElementwiseMulDeviceInput",
    "CudaElementwiseAddDeviceInput", "CudaSoftmax", "CudaEmbeddingLookupDeviceWeight",
    "CudaRopeDeviceInput", "CudaArgMax", "CudaKvCache", "CudaAttentionDecodeDeviceInput",
    "QMatrix", "CudaModel", "Context", "Batch", "ForwardToken", "configs", "tp_plan", "nccl_unique_id",
]


def _torch():
    import torch  # device memory and streams only

    return torch


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    torch = _torch()
    if stream is None:
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return ctypes.c_void_p(stream)


def CudaQuantBuilt() -> bool:
    """CudaQuantBuilt (include/mini_llama/cuda_quant.h:10)."""
    return bool(lib().mlb_built())


def CudaDeviceCount() -> int:
    """CudaDeviceCount (include/mini_llama/cuda_runtime.h:27)."""
    n = ctypes.c_int(0)
    check(lib().mlb_device_count(ctypes.byref(n)))
    return n.value


# ------------------------------------------------------------------ linear

def wait_selftest(which: int, limit_ms: float = 1.0, device_id: int = 0):
    """Runs one of the step kernel's bounded waits against something that
    never arrives (0: a ring slot's mbarrier, 1: a grid barrier) and returns
    the (status code, site) it recorded: (MLB_ERR_TIMEOUT, 900 + which) when
    the wait gave up after limit_ms."""
    code, where = ctypes.c_int(0), ctypes.c_int(0)
    check(lib().mlb_wait_selftest(device_id, which, float(limit_ms), ctypes.byref(code),
                                  ctypes.byref(where)))
    return code.value, where.value


def _linear_device_input(qtype, x, w_dev, block_count, weight_shape, device_id, stream=None):
    torch = _torch()
    if len(weight_shape) != 2:
        raise MlbError(-1, "expected weight shape [out_features, in_features]")
    out_f, in_f = int(weight_shape[0]), int(weight_shape[1])
    if x.dim() not in (1, 2):
        raise MlbError(-1, "expected x shape [in_features] or [batch, in_features]")
    if x.shape[-1] != in_f:
        raise MlbError(-1, f"dimension mismatch x={list(x.shape)} weight=[{out_f}, {in_f}]")
    rows = 1 if x.dim() == 1 else x.shape[0]
    x = x.contiguous()
    y = torch.empty((out_f,) if x.dim() == 1 else (rows, out_f), dtype=torch.float32,
                    device=x.device)
    check(lib().mlb_linear(qtype, _ptr(x), rows, in_f, _ptr(w_dev), block_count, out_f, _ptr(y),
                           device_id, _stream(stream)))
    return y


def CudaQ80LinearDeviceInput(x, w_dev, block_count, weight_shape, device_id=0, stream=None):
    """CudaQ80LinearDeviceInput (include/mini_llama/cuda_quant.h:18)."""
    return _linear_device_input(Q8_0, x, w_dev, block_count, weight_shape, device_id, stream)


def CudaQ40LinearDeviceInput(x, w_dev, block_count, weight_shape, device_id=0, stream=None):
    """CudaQ40LinearDeviceInput (include/mini_llama/cuda_quant.h:24)."""
    return _linear_device_input(Q4_0, x, w_dev, block_count, weight_shape, device_id, stream)


def CudaQ41LinearDeviceInput(x, w_dev, block_count, weight_shape, device_id=0, stream=None):
    """CudaQ41LinearDeviceInput (include/mini_llama/cuda_quant.h:30), with the CPU
    path's d*q + m dequantisation (src/quant.cc:455)."""
    return _linear_device_input(Q4_1, x, w_dev, block_count, weight_shape, device_id, stream)


def CudaLinearDeviceInput(x, w_dev, weight_shape, device_id=0, stream=None):
    """CudaLinearDeviceInput (include/mini_llama/cuda_matmul.h:18), F32 weights."""
    return _linear_device_input(F32, x, w_dev, int(weight_shape[0]) * int(weight_shape[1]),
                                weight_shape, device_id, stream)


def _linear_host(qtype, x, blocks, weight_shape, bias, device_id):
    x = np.ascontiguousarray(x, np.float32)
    blocks = np.ascontiguousarray(blocks)
    out_f, in_f = int(weight_shape[0]), int(weight_shape[1])
    rows = 1 if x.ndim == 1 else x.shape[0]
    nblk = out_f * in_f if qtype == F32 else out_f * ((in_f + 31) // 32)
    y = np.zeros((rows, out_f), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    check(lib().mlb_linear_host(qtype, x.ctypes.data, rows, in_f, blocks.ctypes.data, nblk, out_f,
                                None if b is None else b.ctypes.data, y.ctypes.data, device_id))
    return y[0] if x.ndim == 1 else y


def CudaQ80Linear(x, blocks, weight_shape, bias=None, device_id=0):
    """CudaQ80Linear (include/mini_llama/cuda_quant.h:12): host in, host out."""
    return _linear_host(Q8_0, x, blocks, weight_shape, bias, device_id)


def CudaQ40Linear(x, blocks, weight_shape, bias=None, device_id=0):
    """CudaQ40Linear (include/mini_llama/cuda_quant.h:20)."""
    return _linear_host(Q4_0, x, blocks, weight_shape, bias, device_id)


def CudaQ41Linear(x, blocks, weight_shape, bias=None, device_id=0):
    """CudaQ41Linear (include/mini_llama/cuda_quant.h:26)."""
    return _linear_host(Q4_1, x, blocks, weight_shape, bias, device_id)


def CudaLinear(x, weight, bias=None, device_id=0):
    """CudaLinear (include/mini_llama/cuda_matmul.h:14): F32 weight [out, in]."""
    weight = np.ascontiguousarray(weight, np.float32)
    return _linear_host(F32, x, weight, weight.shape, bias, device_id)


# ------------------------------------------------------------- elementwise

def _empty_like(x):
    return _torch().empty_like(x)


def CudaRmsNormDeviceWeight(x, w, eps, device_id=0, stream=None):
    """CudaRmsNormDeviceWeight (include/mini_llama/cuda_ops.h:27)."""
    if x.dim() != 1 or w.dim() != 1:
        raise MlbError(-1, "RmsNorm: expected 1D tensors")
    if x.shape[0] != w.shape[0]:
        raise MlbError(-1, "RmsNorm: dimension mismatch")
    y = _empty_like(x)
    check(lib().mlb_rmsnorm(_ptr(x), _ptr(w), x.numel(), eps, _ptr(y), device_id, _stream(stream)))
    return y


def CudaSiluDeviceInput(x, device_id=0, stream=None):
    """CudaSiluDeviceInput (include/mini_llama/cuda_ops.h:29)."""
    y = _empty_like(x)
    check(lib().mlb_silu(_ptr(x), x.numel(), _ptr(y), device_id, _stream(stream)))
    return y


def CudaElementwiseMulDeviceInput(a, b, device_id=0, stream=None):
    """CudaElementwiseMulDeviceInput (include/mini_llama/cuda_ops.h:31)."""
    if a.shape != b.shape:
        raise MlbError(-1, f"ElementwiseMul: shape mismatch {list(a.shape)} vs {list(b.shape)}")
    y = _empty_like(a)
    check(lib().mlb_mul(_ptr(a), _ptr(b), a.numel(), _ptr(y), device_id, _stream(stream)))
    return y


def CudaElementwiseAddDeviceInput(a, b, device_id=0, stream=None):
    """CudaElementwiseAddDeviceInput (include/mini_llama/cuda_ops.h:33)."""
    if a.numel() != b.numel():
        raise MlbError(-1, f"ElementwiseAdd: shape mismatch {list(a.shape)} vs {list(b.shape)}")
    y = _empty_like(a)
    check(lib().mlb_add(_ptr(a), _ptr(b), a.numel(), _ptr(y), device_id, _stream(stream)))
    return y


def CudaSoftmax(x, device_id=0, stream=None):
    """CudaSoftmax (include/mini_llama/cuda_ops.h:19) on device data."""
    if x.dim() != 1:
        raise MlbError(-1, "Softmax: expected 1D tensor")
    y = _empty_like(x)
    check(lib().mlb_softmax(_ptr(x), x.numel(), _ptr(y), device_id, _stream(stream)))
    return y


def CudaEmbeddingLookupDeviceWeight(table, token_id, device_id=0, stream=None):
    """CudaEmbeddingLookupDeviceWeight (include/mini_llama/cuda_ops.h:23)."""
    vocab, dim = table.shape
    y = _torch().empty(dim, dtype=table.dtype, device=table.device)
    check(lib().mlb_embedding(_ptr(table), vocab, dim, int(token_id), _ptr(y), device_id,
                              _stream(stream)))
    return y


def CudaRopeDeviceInput(q, k, n_heads, n_kv_heads, head_dim, pos, theta,
                        rope_type=ROPE_NORMAL, device_id=0, stream=None):
    """CudaRopeDeviceInput (include/mini_llama/cuda_ops.h:37): in place."""
    check(lib().mlb_rope(_ptr(q), _ptr(k), n_heads, n_kv_heads, head_dim, pos, theta, rope_type,
                         device_id, _stream(stream)))


def CudaArgMax(x, device_id=0, stream=None) -> int:
    """ArgMax (src/ops.cc:220) on device logits; lowest index wins ties."""
    out = ctypes.c_int(0)
    check(lib().mlb_argmax(_ptr(x), x.numel(), ctypes.byref(out), device_id, _stream(stream)))
    return out.value


# -------------------------------------------------------- KV cache, attention

class CudaKvCache:
    """CudaKvCache (include/mini_llama/cuda_kv_cache.h:9-57): fp32 keys and values
    [n_layers, max_seq_len, n_kv_heads, head_dim] on one device."""

    def __init__(self, n_layers=0, max_seq_len=0, n_kv_heads=0, head_dim=0, device_id=0):
        self.keys = self.values = None
        self._shape = (0, 0, 0, 0)
        self.device_id = device_id
        if n_layers:
            self.Reset(n_layers, max_seq_len, n_kv_heads, head_dim, device_id)

    def Reset(self, n_layers, max_seq_len, n_kv_heads, head_dim, device_id=0):
        torch = _torch()
        for name, v in (("n_layers", n_layers), ("max_seq_len", max_seq_len),
                        ("n_kv_heads", n_kv_heads), ("head_dim", head_dim)):
            if v <= 0:
                raise MlbError(-1, f"CudaKvCache: {name} must be positive")
        self.device_id = device_id
        self._shape = (n_layers, max_seq_len, n_kv_heads, head_dim)
        dev = torch.device("cuda", device_id)
        self.keys = torch.zeros(self._shape, dtype=torch.float32, device=dev)
        self.values = torch.zeros(self._shape, dtype=torch.float32, device=dev)

    def Clear(self):
        if self.keys is not None:
            self.keys.zero_()
            self.values.zero_()

    def empty(self):
        return self.keys is None

    def n_layers(self):
        return self._shape[0]

    def max_seq_len(self):
        return self._shape[1]

    def n_kv_heads(self):
        return self._shape[2]

    def head_dim(self):
        return self._shape[3]

    def bytes(self):
        return 0 if self.keys is None else self.keys.numel() * 4

    def WriteDevice(self, layer, pos, k, v, stream=None):
        L, S, KV, D = self._shape
        check(lib().mlb_kv_write(_ptr(self.keys) if self.keys is not None else None,
                                 _ptr(self.values) if self.values is not None else None,
                                 L, S, KV, D, layer, pos, _ptr(k.contiguous()),
                                 _ptr(v.contiguous()), self.device_id, _stream(stream)))

    def ReadKeyHead(self, layer, pos, kv_head):
        return self.keys[layer, pos, kv_head].cpu().numpy()

    def ReadValueHead(self, layer, pos, kv_head):
        return self.values[layer, pos, kv_head].cpu().numpy()


def CudaAttentionDecodeDeviceInput(q, kv_cache: CudaKvCache, layer, pos, n_heads, n_kv_heads,
                                   head_dim, device_id=0, mode=ATTN_STANDARD, stream=None):
    """CudaAttentionDecodeDeviceInput (include/mini_llama/cuda_attention.h:13).
    mode ATTN_STANDARD matches the reference GPU kernel; ATTN_CPU_COMPAT the CPU path."""
    torch = _torch()
    if q.numel() != n_heads * head_dim:
        raise MlbError(-1, "CudaAttentionDecodeDeviceInput: q shape mismatch")
    if kv_cache.empty():
        raise MlbError(-1, "CudaAttentionDecodeDeviceInput: CUDA KV cache is empty")
    if kv_cache.n_kv_heads() != n_kv_heads or kv_cache.head_dim() != head_dim:
        raise MlbError(-1, "CudaAttentionDecodeDeviceInput: KV cache shape or device does not "
                           "match attention shape")
    out = torch.empty(n_heads * head_dim, dtype=torch.float32, device=q.device)
    L, S, _, _ = kv_cache._shape
    check(lib().mlb_attention_decode(_ptr(q.contiguous()), _ptr(kv_cache.keys),
                                     _ptr(kv_cache.values), L, S, layer, pos, n_heads, n_kv_heads,
                                     head_dim, mode, _ptr(out), device_id, _stream(stream)))
    return out


# ------------------------------------------------------ prepared weight GEMV

class QMatrix:
    """A weight repacked into the B200 GEMV layout (the decode path's format)."""

    def __init__(self, handle, qtype, out_features, in_features, device_id=0):
        self.h = handle
        self.qtype, self.out_features, self.in_features = qtype, out_features, in_features
        self.device_id = device_id

    @classmethod
    def from_gguf(cls, qtype, blocks, out_features, in_features, device_id=0):
        """blocks: host numpy uint8/float32 array, or a CUDA tensor, in GGUF layout."""
        h = ctypes.c_void_p()
        if isinstance(blocks, np.ndarray):
            blocks = np.ascontiguousarray(blocks)
            check(lib().mlb_qmatrix_create(qtype, blocks.ctypes.data, 1, out_features, in_features,
                                           device_id, ctypes.byref(h)))
        else:
            check(lib().mlb_qmatrix_create(qtype, _ptr(blocks), 0, out_features, in_features,
                                           device_id, ctypes.byref(h)))
        return cls(h, qtype, out_features, in_features, device_id)

    @classmethod
    def synthesize(cls, qtype, out_features, in_features, seed, stream_id=0, raw=False,
                   device_id=0):
        h = ctypes.c_void_p()
        check(lib().mlb_qmatrix_synthesize(qtype, out_features, in_features, seed, stream_id,
                                           int(raw), device_id, ctypes.byref(h)))
        return cls(h, qtype, out_features, in_features, device_id)

    def gemv(self, x, y=None, stream=None):
        torch = _torch()
        rows = 1 if x.dim() == 1 else x.shape[0]
        if y is None:
            y = torch.empty((rows, self.out_features) if x.dim() == 2 else (self.out_features,),
                            dtype=torch.float32, device=x.device)
        check(lib().mlb_qmatrix_gemv(self.h, _ptr(x), rows, _ptr(y), _stream(stream)))
        return y

    def gemm(self, x, y=None, stream=None):
        """y = W x on the tensor cores (mlb_qmatrix_gemm), any row count."""
        torch = _torch()
        rows = 1 if x.dim() == 1 else x.shape[0]
        if y is None:
            y = torch.empty((rows, self.out_features) if x.dim() == 2 else (self.out_features,),
                            dtype=torch.float32, device=x.device)
        check(lib().mlb_qmatrix_gemm(self.h, _ptr(x), rows, _ptr(y), _stream(stream)))
        return y

    def dequant(self, out=None, stream=None):
        """fp32 [out_features, in_features] on the device, decoded from the
        repacked layout (DequantizeFromQ80/Q40/Q41, src/quant.cc:170-361)."""
        torch = _torch()
        if out is None:
            out = torch.empty((self.out_features, self.in_features), dtype=torch.float32,
                              device=f"cuda:{self.device_id}")
        check(lib().mlb_qmatrix_dequant(self.h, _ptr(out), _stream(stream)))
        return out

    def gguf_bytes(self):
        return lib().mlb_qmatrix_bytes(self.h)

    def __del__(self):
        try:
            if self.h:
                lib().mlb_qmatrix_destroy(self.h)
                self.h = None
        except Exception:
            pass


# ------------------------------------------------------------ model, context

class CudaModel:
    """Device-resident model: UploadModelWeightsToCuda (src/model.cc:345-374) as
    set_weight/finalize, or seeded on-device synthesis. tp_size > 1 keeps this
    rank's tensor-parallel shard (nccl_id: 128 bytes from nccl_unique_id())."""

    def __init__(self, cfg: dict, device_id=0, tp_rank=0, tp_size=1, nccl_id: bytes | None = None):
        self.cfg = dict(cfg)
        self.device_id = device_id
        c = MlbConfig(**{k: cfg[k] for k, _ in MlbConfig._fields_})
        h = ctypes.c_void_p()
        idbuf = None if nccl_id is None else ctypes.create_string_buffer(bytes(nccl_id), 128)
        check(lib().mlb_model_create(ctypes.byref(c), device_id, tp_rank, tp_size, idbuf,
                                     ctypes.byref(h)))
        self.h = h

    @classmethod
    def from_gguf(cls, path: str, device_id=0, tp_rank=0, tp_size=1, nccl_id: bytes | None = None,
                  max_seq_len: int = 0):
        """LoadGgufModel + UploadModelWeightsToCuda (mlb_model_load_gguf): the model
        of a GGUF v3 file, uploaded from the mapped file and finalized.
        max_seq_len > 0 replaces the file's context_length. The bytes copied to
        the device are in .gguf_bytes."""
        self = cls.__new__(cls)
        self.cfg = read_gguf_config(path)
        if max_seq_len > 0:
            self.cfg["max_seq_len"] = max_seq_len
        self.device_id = device_id
        h = ctypes.c_void_p()
        n = ctypes.c_size_t()
        idbuf = None if nccl_id is None else ctypes.create_string_buffer(bytes(nccl_id), 128)
        check(lib().mlb_model_load_gguf(os.fsencode(path), device_id, tp_rank, tp_size, idbuf,
                                        int(max_seq_len), ctypes.byref(h), ctypes.byref(n)))
        self.h = h
        self.gguf_bytes = n.value
        return self

    def set_weight(self, kind, layer, qtype, rows, cols, data: np.ndarray):
        data = np.ascontiguousarray(data)
        check(lib().mlb_model_set_weight(self.h, kind, layer, qtype, rows, cols, data.ctypes.data,
                                         data.nbytes))

    def load(self, weights):
        """weights: iterable of (kind, layer, qtype, rows, cols, array)."""
        for kind, layer, qtype, rows, cols, arr in weights:
            self.set_weight(kind, layer, qtype, rows, cols, arr)
        self.finalize()
        return self

    def synthesize(self, qtype, seed, with_bias=False):
        check(lib().mlb_model_synthesize(self.h, qtype, seed, int(with_bias)))
        return self

    def finalize(self):
        check(lib().mlb_model_finalize(self.h))
        return self

    def bytes(self):
        r, s = ctypes.c_size_t(), ctypes.c_size_t()
        check(lib().mlb_model_bytes(self.h, ctypes.byref(r), ctypes.byref(s)))
        return r.value, s.value

    def context(self, attention_mode=ATTN_CPU_COMPAT, step_kernel=None, kv_type=0):
        return Context(self, attention_mode, step_kernel, kv_type)

    def close(self):
        if getattr(self, "h", None):
            lib().mlb_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Context:
    """MiniLlamaContext with its CUDA KV cache (include/mini_llama/context.h)."""

    def __init__(self, model: CudaModel, attention_mode=ATTN_CPU_COMPAT, step_kernel=None,
                 kv_type: int = 0):
        """kv_type: KV_F32 (the reference's fp32 cache) or KV_BF16 (step kernel only)."""
        self.model = model
        h = ctypes.c_void_p()
        check(lib().mlb_context_create_kv(model.h, attention_mode, int(kv_type), ctypes.byref(h)))
        self.h = h
        self.pos = 0
        self.token_history = []
        if step_kernel is not None:
            self.set_step_kernel(step_kernel)

    def set_step_kernel(self, enable: bool):
        """True: one persistent kernel per decode step; False: one kernel per op."""
        check(lib().mlb_context_set_step_kernel(self.h, 1 if enable else 0))

    def step_kernel(self) -> bool:
        return bool(lib().mlb_context_step_kernel(self.h))

    def decode_sample(self, sampler: "Sampler", token: int, pos: int, n_steps: int,
                      temperature: float = 0.0, top_k: int = 0) -> list:
        """decode_greedy with the sampler's choice at every step (mlb_decode_sample)."""
        out = np.empty(max(n_steps, 1), np.int32)
        check(lib().mlb_decode_sample(self.h, sampler.h, float(temperature), int(top_k),
                                      int(token), int(pos), int(n_steps), out.ctypes.data))
        return [int(t) for t in out[:n_steps]]

    def step_trace(self, enable: bool):
        """Records per-phase times of later step-kernel steps (diagnostic)."""
        check(lib().mlb_context_step_trace(self.h, 1 if enable else 0))

    def step_trace_read(self) -> np.ndarray:
        """Global-timer stamps (ns) of the last traced step, [phase][cta][2]:
        start of each phase's work after its barrier, end before the next.
        Phases: per layer QKV, attention, wo, gate/up, w_down; then lm_head."""
        n, g = ctypes.c_int(0), ctypes.c_int(0)
        check(lib().mlb_context_step_trace_read(self.h, None, 0, ctypes.byref(n),
                                                ctypes.byref(g)))
        out = np.zeros((n.value, g.value, 2), np.uint64)
        check(lib().mlb_context_step_trace_read(self.h, out.ctypes.data, out.size,
                                                ctypes.byref(n), ctypes.byref(g)))
        return out

    def forward_token(self, token: int, pos: int) -> np.ndarray:
        """ForwardToken's device branch (src/forward.cc:776-794): host logits."""
        out = np.empty(self.model.cfg["vocab_size"], np.float32)
        check(lib().mlb_forward_token(self.h, int(token), int(pos), out.ctypes.data))
        return out

    def forward_token_device(self, token: int, pos: int) -> int:
        """Asynchronous step; returns the device address of the logits."""
        p = ctypes.c_void_p()
        check(lib().mlb_forward_token_device(self.h, int(token), int(pos), ctypes.byref(p)))
        return p.value

    def sync(self):
        check(lib().mlb_context_sync(self.h))

    def decode_greedy(self, token: int, pos: int, n_steps: int) -> list:
        out = np.empty(max(n_steps, 1), np.int32)
        check(lib().mlb_decode_greedy(self.h, int(token), int(pos), int(n_steps), out.ctypes.data))
        return [int(t) for t in out[:n_steps]]

    def reset(self):
        check(lib().mlb_context_reset(self.h))
        self.pos = 0
        self.token_history = []

    def fill_kv(self, n_pos: int, seed: int, scale: float = 1.25):
        """Seeded K/V rows for positions [0, n_pos) (mlb_context_fill_kv)."""
        check(lib().mlb_context_fill_kv(self.h, int(n_pos), int(seed), float(scale)))

    def forward_batch(self, tokens, positions) -> np.ndarray:
        """ForwardBatch (src/batch.cc:35-50): every token at its position, the
        last token's logits (mlb_forward_batch)."""
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        out = np.empty(self.model.cfg["vocab_size"], np.float32)
        check(lib().mlb_forward_batch(self.h, len(t), t.ctypes.data, p.ctypes.data,
                                      out.ctypes.data))
        return out

    def stream(self) -> int:
        return lib().mlb_context_stream(self.h) or 0

    def kernels_per_step(self) -> int:
        return lib().mlb_context_kernels_per_step(self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().mlb_context_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Sampler:
    """MiniSampler (include/mini_llama/sampler.h) on the device: a std::mt19937
    seeded with `seed` (0: a random seed) whose state stays on device_id."""

    def __init__(self, seed: int = 0, device_id: int = 0):
        h = ctypes.c_void_p()
        check(lib().mlb_sampler_create(int(device_id), int(seed), ctypes.byref(h)))
        self.h = h
        self.device_id = device_id

    def sample(self, logits_ptr: int, n: int, temperature: float = 0.0, top_k: int = 0) -> int:
        """MiniSampler::Sample over n fp32 logits at device address logits_ptr."""
        out = ctypes.c_int(-1)
        check(lib().mlb_sample(self.h, ctypes.c_void_p(logits_ptr), int(n), float(temperature),
                               int(top_k), ctypes.byref(out)))
        return out.value

    def close(self):
        if getattr(self, "h", None):
            lib().mlb_sampler_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Batch:
    """n_seqs sequences decoded together (mlb_batch_*), each with its own KV cache."""

    def __init__(self, model: CudaModel, n_seqs: int, attention_mode=ATTN_CPU_COMPAT,
                 kv_type: int = 0):
        """kv_type: KV_F32 (the reference's fp32 cache) or KV_BF16."""
        self.model = model
        self.n_seqs = n_seqs
        self.kv_type = kv_type
        h = ctypes.c_void_p()
        check(lib().mlb_batch_create_kv(model.h, int(n_seqs), attention_mode, int(kv_type),
                                        ctypes.byref(h)))
        self.h = h

    def reset(self):
        check(lib().mlb_batch_reset(self.h))

    def fill_kv(self, seq: int, n_pos: int, seed: int, scale: float = 1.25):
        check(lib().mlb_batch_fill_kv(self.h, int(seq), int(n_pos), int(seed), float(scale)))

    def forward(self, seqs, tokens, positions, logits=False):
        """One pass of rows; returns (next greedy ids, logits [rows, vocab] or None)."""
        s = np.ascontiguousarray(seqs, np.int32)
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        nxt = np.empty(len(t), np.int32)
        lg = np.empty((len(t), self.model.cfg["vocab_size"]), np.float32) if logits else None
        check(lib().mlb_batch_forward(self.h, len(t), s.ctypes.data, t.ctypes.data, p.ctypes.data,
                                      lg.ctypes.data if logits else None, nxt.ctypes.data))
        return [int(v) for v in nxt], lg

    def decode_greedy(self, tokens, positions, n_steps: int) -> np.ndarray:
        """[n_steps, n_seqs] greedy ids, all sequences in lockstep."""
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        out = np.empty((max(n_steps, 1), self.n_seqs), np.int32)
        check(lib().mlb_batch_decode_greedy(self.h, t.ctypes.data, p.ctypes.data, int(n_steps),
                                            out.ctypes.data))
        return out[:n_steps]

    def stream(self) -> int:
        return lib().mlb_batch_stream(self.h) or 0

    def kernels_per_step(self) -> int:
        return lib().mlb_batch_kernels_per_step(self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().mlb_batch_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ForwardToken(ctx: Context, token: int) -> np.ndarray:
    """ForwardToken(ctx, model, token) (include/mini_llama/forward.h:11) at ctx.pos."""
    return ctx.forward_token(token, ctx.pos)


def read_gguf_config(path: str) -> dict:
    """The model config LoadGgufModel builds from a GGUF file (host only)."""
    c = MlbConfig()
    check(lib().mlb_gguf_read_config(os.fsencode(path), ctypes.byref(c)))
    return {k: getattr(c, k) for k, _ in MlbConfig._fields_}


def tp_plan(cfg: dict, tp_rank: int, tp_size: int) -> dict:
    """The tensor-parallel shard of one rank (host only; see mlb_tp_plan)."""
    from ._lib import MlbTpShard

    c = MlbConfig(**{k: cfg[k] for k, _ in MlbConfig._fields_})
    out = MlbTpShard()
    check(lib().mlb_tp_plan(ctypes.byref(c), int(tp_rank), int(tp_size), ctypes.byref(out)))
    return {k: getattr(out, k) for k, _ in MlbTpShard._fields_}


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    check(lib().mlb_nccl_unique_id(buf))
    return buf.raw
