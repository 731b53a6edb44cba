"""The seeded weight generator and the C ABI library (CPU-only checks)."""
import ctypes
import json
import os
import re

import numpy as np
import pytest

from tests.conftest import ROOT, golden_path
from mini_llama_b200 import _lib
from mini_llama_b200 import configs as C


def test_generator_quantizers_match_reference_bits(port, ref):
    s = _lib.synth_lib()
    rng = np.random.default_rng(11)
    for trial in range(40):
        n = 32 if trial % 4 else int(rng.integers(1, 32))
        x = (rng.normal(0, 0.02 * (1 + trial % 5), n)).astype(np.float32)
        if trial % 7 == 0:
            x[:] = 0
        for qtype in (C.Q8_0, C.Q4_0, C.Q4_1):
            out = np.zeros(C.BLOCK_BYTES[qtype], np.uint8)
            s.mlbs_quantize_block(qtype, x.ctypes.data, n, out.ctypes.data)
            np.testing.assert_array_equal(out, port.quantize(qtype, x[None]))
            if qtype != C.Q4_1:
                np.testing.assert_array_equal(out, ref.quantize(qtype, x[None]))


def test_generator_fp16_matches_reference_rounding(port):
    s = _lib.synth_lib()
    rng = np.random.default_rng(5)
    vals = np.concatenate([rng.normal(0, 1, 2000), rng.normal(0, 1e-5, 500),
                           rng.normal(0, 1e5, 100)]).astype(np.float32)
    for v in vals:
        assert s.mlbs_f32_to_fp16(float(v)) == port.f32_to_fp16(float(v))


def test_generator_is_deterministic_and_pinned():
    meta = json.load(open(golden_path("golden.json")))
    from tests.golden.make_golden import weights_digest  # same digest as the fixtures

    for name in ("small_q4_0_gqa", "small_q4_1_neox_bias", "small_q8_0_ragged"):
        m = meta[name]
        qtype = {v: k for k, v in C.QTYPE_NAMES.items()}[m["qtype"]]
        ws = list(C.host_weights(m["config"], qtype, m["seed"], m["bias"], threads=3))
        assert weights_digest(ws) == m["weights_sha256"], name


def test_generator_statistics():
    emb = C.synth_tensor(3, C.W_TOKEN_EMBEDDING, -1, C.F32, 256, 512)
    assert abs(float(emb.mean())) < 1e-3
    assert abs(float(emb.std()) - 0.02) < 5e-4
    a = C.synth_tensor(3, C.W_WQ, 0, C.Q4_0, 64, 256)
    b = C.synth_tensor(3, C.W_WQ, 1, C.Q4_0, 64, 256)
    assert not np.array_equal(a, b)  # streams differ per layer


def _header_functions():
    text = open(os.path.join(ROOT, "include", "mlb200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mlb_[a-z0-9_]+)\s*\(", text)))


def test_c_abi_exports_every_declared_symbol():
    path = os.path.join(ROOT, "mini_llama_b200", "libmlb200.so")
    if not os.path.exists(path):
        from mini_llama_b200 import build

        build.build_cuda()
    lib = ctypes.CDLL(path)
    names = _header_functions()
    assert len(names) >= 30
    for n in names:
        assert hasattr(lib, n), n
    bound = {s[0] for s in _lib.SIGNATURES}
    assert set(names) == bound


def test_c_abi_reports_errors_without_a_gpu():
    lib = _lib.lib()
    n = ctypes.c_int(-1)
    assert lib.mlb_device_count(ctypes.byref(n)) == 0
    rc = lib.mlb_linear(C.Q4_0, None, 1, 64, None, 7, 4, None, 0, None)
    assert rc == -1
    assert b"block count mismatch" in lib.mlb_last_error()
    assert lib.mlb_built() == 1


@pytest.mark.parametrize("name,cfg_q", list(C.WORKLOADS.items()))
def test_workload_shapes_are_block_aligned(name, cfg_q):
    cfg, qtype, bias = cfg_q
    assert cfg["dim"] % 32 == 0 and cfg["hidden_dim"] % 32 == 0
    assert cfg["n_heads"] % cfg["n_kv_heads"] == 0
    assert cfg["n_heads"] * cfg["head_dim"] == cfg["dim"]


def test_c_abi_rejects_injected_faults_without_touching_a_device():
    """Host-side fault injection through the C ABI: every bad argument returns
    an error status with the reference's kind of message, before any device
    call (so it runs with no GPU)."""
    lib = _lib.lib()
    bad = ctypes.c_void_p(1)  # never dereferenced: the checks come first

    def err(rc, text, code=-1):
        assert rc == code, (rc, lib.mlb_last_error())
        assert text.encode() in lib.mlb_last_error(), lib.mlb_last_error()

    err(lib.mlb_linear(99, bad, 1, 64, bad, 2, 1, bad, 0, None), "unsupported quant type 99")
    err(lib.mlb_linear(C.Q8_0, bad, 0, 64, bad, 2, 1, bad, 0, None), "empty tensors")
    err(lib.mlb_linear(C.Q4_0, bad, 1, 64, bad, 3, 1, bad, 0, None), "block count mismatch")
    err(lib.mlb_linear(C.Q4_0, None, 1, 64, bad, 2, 1, bad, 0, None), "pointer is null")
    err(lib.mlb_qmatrix_gemv(None, bad, 1, bad, None), "null pointer")
    cfg = _lib.MlbConfig(vocab_size=10, dim=64, hidden_dim=96, n_layers=1, n_heads=4,
                         n_kv_heads=3, head_dim=16, max_seq_len=8, rope_theta=1e4,
                         rms_norm_eps=1e-5, rope_type=0)
    out = ctypes.c_void_p()
    err(lib.mlb_model_create(ctypes.byref(cfg), 0, 0, 1, None, ctypes.byref(out)),
        "n_heads must be divisible by n_kv_heads")
    cfg.n_kv_heads, cfg.dim = 2, 0
    err(lib.mlb_model_create(ctypes.byref(cfg), 0, 0, 1, None, ctypes.byref(out)),
        "config dimensions must be positive")
    cfg.dim, cfg.head_dim = 64, 18
    err(lib.mlb_model_create(ctypes.byref(cfg), 0, 0, 1, None, ctypes.byref(out)),
        "head_dim must be a multiple of 4")
    cfg.head_dim = 16
    err(lib.mlb_model_create(ctypes.byref(cfg), 0, 2, 2, None, ctypes.byref(out)),
        "bad tensor-parallel rank/size")
    err(lib.mlb_model_create(None, 0, 0, 1, None, ctypes.byref(out)), "null config")
    err(lib.mlb_forward_token(None, 1, 0, bad), "null pointer")
    err(lib.mlb_context_sync(None), "null context")
    err(lib.mlb_context_set_step_kernel(None, 1), "null context")
    code, where = ctypes.c_int(0), ctypes.c_int(0)
    err(lib.mlb_wait_selftest(0, 2, 1.0, ctypes.byref(code), ctypes.byref(where)),
        "which must be 0 or 1")
