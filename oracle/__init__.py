"""CPU oracles for the decode forward path — TEST INFRASTRUCTURE ONLY.

Two oracles, both loaded with ctypes:

* ``port`` — oracle/libmlport.so, a C restatement of the reference's CPU
  algorithm (oracle/port/mlport.c; each function cites the reference
  file:line it follows).
* ``ref``  — oracle/_ref/libmlref.so, the reference's own unmodified CPU
  sources compiled in place plus oracle/ref_shim.cc. Present only where it
  was built (it needs the reference tree at build time); ``ref_available()``
  says whether it loaded.

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs import this
package. The product library (mini_llama_b200) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "libmlport.so")
REF_SO = os.path.join(HERE, "_ref", "libmlref.so")

F32, Q8_0, Q4_0, Q4_1 = 0, 1, 2, 3
BLOCK_BYTES = {Q8_0: 34, Q4_0: 18, Q4_1: 20}

_f = ctypes.POINTER(ctypes.c_float)
_vp = ctypes.c_void_p


def build(ref: bool = True) -> None:
    """Build the port (always) and the reference shim (when the reference tree
    is found: $REF_ROOT, else the checkout named `reference` beside this
    repository)."""
    targets = ["port"] + (["ref-if-present"] if ref else [])
    args = []
    if ref:
        root = os.environ.get("REF_ROOT") or os.path.join(
            os.path.dirname(os.path.dirname(HERE.rstrip(os.sep))), "reference")
        args = [f"REF_ROOT={root}"]
    subprocess.run(["make", "-s", "-C", HERE] + targets + args, check=True)


def weight_bytes(qtype: int, rows: int, cols: int) -> int:
    if qtype == F32:
        return rows * cols * 4
    return rows * ((cols + 31) // 32) * BLOCK_BYTES[qtype]


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_vp)


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(_f)


class _Lib:
    """Common wrappers; prefix is 'mlp_' (port) or 'ref_' (reference)."""

    def __init__(self, path: str, prefix: str):
        self.lib = ctypes.CDLL(path)
        self.p = prefix
        L = self.lib
        g = lambda n: getattr(L, prefix + n)
        g("linear").argtypes = [ctypes.c_int, _f, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, _f]
        g("dequant").argtypes = [ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, _f]
        g("quantize").argtypes = [ctypes.c_int, _f, ctypes.c_int, ctypes.c_int, _vp]
        g("rmsnorm").argtypes = [_f, _f, ctypes.c_int, ctypes.c_float, _f]
        g("softmax").argtypes = [_f, ctypes.c_int, _f]
        g("swiglu").argtypes = [_f, _f, ctypes.c_int, _f]
        g("rope").argtypes = [_f, ctypes.c_int, _f, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                              ctypes.c_float, ctypes.c_int]
        g("argmax").argtypes = [_f, ctypes.c_int]
        g("last_error").restype = ctypes.c_char_p

    def _g(self, n):
        return getattr(self.lib, self.p + n)

    def _check(self, rc):
        if rc is not None and rc < 0:
            err = self._g("last_error")().decode()
            if rc == -2:
                raise IndexError(err)
            raise RuntimeError(err)
        return rc

    def linear(self, qtype, x, w, out_features):
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows = 1 if x.ndim == 1 else x.shape[0]
        k = x.shape[-1]
        y = np.zeros((rows, out_features), np.float32)
        self._check(self._g("linear")(qtype, _fptr(x), rows, k, _ptr(np.ascontiguousarray(w)),
                                      out_features, _fptr(y)))
        return y[0] if x.ndim == 1 else y

    def dequant(self, qtype, w, rows, cols):
        out = np.zeros((rows, cols), np.float32)
        self._check(self._g("dequant")(qtype, _ptr(np.ascontiguousarray(w)), rows, cols, _fptr(out)))
        return out

    def quantize(self, qtype, src):
        src = np.ascontiguousarray(src, dtype=np.float32)
        rows, cols = src.shape
        out = np.zeros(weight_bytes(qtype, rows, cols), np.uint8)
        self._check(self._g("quantize")(qtype, _fptr(src), rows, cols, _ptr(out)))
        return out

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros_like(x)
        self._check(self._g("rmsnorm")(_fptr(x), _fptr(np.ascontiguousarray(w, np.float32)),
                                       x.size, eps, _fptr(y)))
        return y

    def softmax(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros_like(x)
        self._check(self._g("softmax")(_fptr(x), x.size, _fptr(y)))
        return y

    def swiglu(self, g, u):
        g = np.ascontiguousarray(g, np.float32)
        y = np.zeros_like(g)
        self._check(self._g("swiglu")(_fptr(g), _fptr(np.ascontiguousarray(u, np.float32)),
                                      g.size, _fptr(y)))
        return y

    def rope(self, q, k, pos, theta, neox):
        q = np.array(q, np.float32, copy=True)
        k = np.array(k, np.float32, copy=True)
        self._check(self._g("rope")(_fptr(q), q.shape[0], _fptr(k), k.shape[0], q.shape[1],
                                    pos, theta, int(neox)))
        return q, k

    def argmax(self, x):
        x = np.ascontiguousarray(x, np.float32)
        return self._g("argmax")(_fptr(x), x.size)


class Port(_Lib):
    """The C restatement (oracle/port/mlport.c)."""

    class Config(ctypes.Structure):
        _fields_ = [(n, ctypes.c_int) for n in ("vocab_size", "dim", "hidden_dim", "n_layers",
                                                 "n_heads", "n_kv_heads", "head_dim",
                                                 "max_seq_len")] + [
            ("rope_theta", ctypes.c_float), ("rms_norm_eps", ctypes.c_float),
            ("rope_type", ctypes.c_int)]

    def __init__(self):
        super().__init__(PORT_SO, "mlp_")
        L = self.lib
        for fn in ("mlp_rmsnorm", "mlp_softmax", "mlp_swiglu", "mlp_rope", "mlp_attention"):
            getattr(L, fn).restype = None  # void in oracle/port/mlport.h
        L.mlp_attention.argtypes = [_f, _f, _f] + [ctypes.c_int] * 7 + [_f]
        L.mlp_attention_scale.argtypes = [ctypes.c_int]
        L.mlp_attention_scale.restype = ctypes.c_float
        L.mlp_f32_to_fp16.argtypes = [ctypes.c_float]
        L.mlp_f32_to_fp16.restype = ctypes.c_uint16
        L.mlp_fp16_to_f32.argtypes = [ctypes.c_uint16]
        L.mlp_fp16_to_f32.restype = ctypes.c_float
        L.mlp_model_create.argtypes = [ctypes.POINTER(Port.Config)]
        L.mlp_model_create.restype = _vp
        L.mlp_model_destroy.argtypes = [_vp]
        L.mlp_model_set_weight.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_int, _vp, ctypes.c_size_t]
        L.mlp_ctx_create.argtypes = [_vp]
        L.mlp_ctx_create.restype = _vp
        L.mlp_ctx_destroy.argtypes = [_vp]
        L.mlp_ctx_set_kv_bf16.argtypes = [_vp, ctypes.c_int]
        L.mlp_ctx_set_kv_bf16.restype = None
        L.mlp_ctx_kv.argtypes = [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp)]
        L.mlp_ctx_kv.restype = None
        L.mlp_forward_token.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _f]

    def attention(self, q, keys, values, layer, pos, n_heads, n_kv_heads, head_dim,
                  include_current_v=False):
        """keys/values: [L, max_seq, KV, D] float32."""
        out = np.zeros((n_heads, head_dim), np.float32)
        self.lib.mlp_attention(_fptr(np.ascontiguousarray(q, np.float32)),
                               _fptr(np.ascontiguousarray(keys, np.float32)),
                               _fptr(np.ascontiguousarray(values, np.float32)),
                               layer, keys.shape[1], n_heads, n_kv_heads, head_dim, pos,
                               int(include_current_v), _fptr(out))
        return out

    def attention_scale(self, head_dim):
        return self.lib.mlp_attention_scale(head_dim)

    def f32_to_fp16(self, v):
        return self.lib.mlp_f32_to_fp16(v)

    def fp16_to_f32(self, h):
        return self.lib.mlp_fp16_to_f32(h)

    def model(self, cfg):
        return PortModel(self, cfg)


class PortModel:
    """A model + context on the C restatement; forward_token mirrors ForwardToken."""

    def __init__(self, port: Port, cfg: dict):
        self.port = port
        self.cfg = dict(cfg)
        c = Port.Config(**{k: cfg[k] for k, _ in Port.Config._fields_})
        self.h = port.lib.mlp_model_create(ctypes.byref(c))
        self.ctx = None

    def set_weight(self, kind, layer, qtype, rows, cols, data: np.ndarray):
        data = np.ascontiguousarray(data)
        self.port._check(self.port.lib.mlp_model_set_weight(
            self.h, kind, layer, qtype, rows, cols, _ptr(data), data.nbytes))

    def _context(self):
        if self.ctx is None:
            self.ctx = self.port.lib.mlp_ctx_create(self.h)
            if not self.ctx:
                raise MemoryError("mlp_ctx_create failed")
        return self.ctx

    def set_kv_bf16(self, on: bool):
        """K and V rounded to bf16 when written (the GPU's bf16 cache option;
        not a reference mode)."""
        self.port.lib.mlp_ctx_set_kv_bf16(self._context(), int(on))

    def kv_cache(self):
        """(keys, values) views [L, max_seq, KV, D] of the context's cache."""
        k, v = _vp(), _vp()
        self.port.lib.mlp_ctx_kv(self._context(), ctypes.byref(k), ctypes.byref(v))
        shape = (self.cfg["n_layers"], self.cfg["max_seq_len"], self.cfg["n_kv_heads"],
                 self.cfg["head_dim"])
        n = int(np.prod(shape))
        as_arr = lambda p: np.ctypeslib.as_array((ctypes.c_float * n).from_address(p.value)).reshape(shape)  # noqa: E731
        return as_arr(k), as_arr(v)

    def forward_token(self, token, pos):
        self._context()
        out = np.zeros(self.cfg["vocab_size"], np.float32)
        self.port._check(self.port.lib.mlp_forward_token(self.ctx, token, pos, _fptr(out)))
        return out

    def __del__(self):
        try:
            if self.ctx:
                self.port.lib.mlp_ctx_destroy(self.ctx)
            self.port.lib.mlp_model_destroy(self.h)
        except Exception:
            pass


class Ref(_Lib):
    """The reference's own CPU code (oracle/_ref/libmlref.so)."""

    def __init__(self):
        super().__init__(REF_SO, "ref_")
        L = self.lib
        L.ref_model_create.argtypes = [ctypes.c_int] * 8 + [ctypes.c_float, ctypes.c_float,
                                                             ctypes.c_int]
        L.ref_model_create.restype = _vp
        L.ref_model_destroy.argtypes = [_vp]
        L.ref_model_load_gguf.argtypes = [ctypes.c_char_p]
        L.ref_model_load_gguf.restype = _vp
        L.ref_model_set_weight.argtypes = [_vp] + [ctypes.c_int] * 5 + [_vp]
        L.ref_model_config.argtypes = [_vp, ctypes.POINTER(ctypes.c_int)]
        L.ref_ctx_create.argtypes = [_vp]
        L.ref_ctx_create.restype = _vp
        L.ref_ctx_destroy.argtypes = [_vp]
        L.ref_forward_token.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _f]
        L.ref_set_threads.argtypes = [ctypes.c_int]
        L.ref_model_synthesize.argtypes = [_vp, ctypes.c_int, ctypes.c_uint64, ctypes.c_int,
                                           ctypes.c_int]
        L.ref_ctx_fill_kv.argtypes = [_vp, ctypes.c_int, ctypes.c_uint64, ctypes.c_float]
        L.ref_sampler_create.argtypes = [ctypes.c_uint]
        L.ref_sampler_create.restype = _vp
        L.ref_sampler_destroy.argtypes = [_vp]
        L.ref_sample.argtypes = [_vp, _f, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                                 ctypes.POINTER(ctypes.c_int)]

    def set_threads(self, n):
        self.lib.ref_set_threads(n)

    def threads(self):
        return self.lib.ref_get_threads()

    def model(self, cfg):
        return RefModel(self, cfg)

    def sampler(self, seed):
        return RefSampler(self, seed)

    def load_gguf(self, path):
        """A model read by the reference's own LoadGgufModel."""
        h = self.lib.ref_model_load_gguf(os.fsencode(path))
        if not h:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return RefModel(self, handle=h)


class RefSampler:
    """A MiniSampler (src/sampler.cc) in the reference's own code."""

    def __init__(self, ref: Ref, seed: int):
        self.ref = ref
        self.h = ref.lib.ref_sampler_create(int(seed))
        if not self.h:
            raise RuntimeError(ref.lib.ref_last_error().decode())

    def sample(self, logits, temperature, top_k):
        x = np.ascontiguousarray(logits, np.float32)
        out = ctypes.c_int(-1)
        self.ref._check(self.ref.lib.ref_sample(self.h, _fptr(x), x.size, float(temperature),
                                                int(top_k), ctypes.byref(out)))
        return out.value

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.ref_sampler_destroy(self.h)
            self.h = None


class RefModel:
    """A MiniLlamaModel + MiniLlamaContext in the reference's own code."""

    def __init__(self, ref: Ref, cfg: dict | None = None, handle=None):
        self.ref = ref
        self.ctx = None
        if handle is not None:
            self.h = handle
            v = (ctypes.c_int * 11)()
            ref.lib.ref_model_config(self.h, v)
            keys = ("vocab_size", "dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads",
                    "head_dim", "max_seq_len")
            self.cfg = {k: v[i] for i, k in enumerate(keys)}
            self.cfg["rope_type"] = v[10]
        else:
            self.cfg = dict(cfg)
            self.h = ref.lib.ref_model_create(*[cfg[k] for k in (
                "vocab_size", "dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads",
                "head_dim", "max_seq_len", "rope_theta", "rms_norm_eps", "rope_type")])

    def set_weight(self, kind, layer, qtype, rows, cols, data: np.ndarray):
        data = np.ascontiguousarray(data)
        self.ref._check(self.ref.lib.ref_model_set_weight(self.h, kind, layer, qtype, rows, cols,
                                                          _ptr(data)))

    def synthesize(self, qtype, seed, with_bias=False, threads=8):
        """Every weight from the seeded generator, quantised with the
        reference's own quantisers (ref_model_synthesize in ref_shim.cc):
        the bytes the GPU library's CudaModel.synthesize generates."""
        self.ref._check(self.ref.lib.ref_model_synthesize(self.h, qtype, seed, int(with_bias),
                                                          threads))
        return self

    def _context(self):
        if self.ctx is None:
            self.ctx = self.ref.lib.ref_ctx_create(self.h)
            if not self.ctx:
                raise RuntimeError(self.ref.lib.ref_last_error().decode())
        return self.ctx

    def new_context(self):
        """Drops the current MiniLlamaContext; the next call makes a fresh one."""
        if self.ctx:
            self.ref.lib.ref_ctx_destroy(self.ctx)
        self.ctx = None

    def fill_kv(self, n_pos, seed, scale=1.25):
        """Seeded K/V rows for positions [0, n_pos) of every layer, written with
        KvCache::Write (the values mlb_context_fill_kv writes on the GPU)."""
        self.ref._check(self.ref.lib.ref_ctx_fill_kv(self._context(), n_pos, seed, scale))

    def forward_token(self, token, pos):
        self._context()
        out = np.zeros(self.cfg["vocab_size"], np.float32)
        self.ref._check(self.ref.lib.ref_forward_token(self.ctx, token, pos, _fptr(out)))
        return out

    def __del__(self):
        try:
            if self.ctx:
                self.ref.lib.ref_ctx_destroy(self.ctx)
            self.ref.lib.ref_model_destroy(self.h)
        except Exception:
            pass


_port = None
_ref = None


def port() -> Port:
    global _port
    if _port is None:
        if not os.path.exists(PORT_SO):
            build(ref=False)
        _port = Port()
    return _port


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref() -> Ref:
    global _ref
    if _ref is None:
        _ref = Ref()
    return _ref
