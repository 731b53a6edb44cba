"""Kernel parity on the GPU, through the C ABI, against the CPU oracle.

Tolerances are the reference's own GPU-vs-CPU conventions: quantised linear
abs <= 1e-3 or rel <= 1e-3 (tests/test_cuda_quant.cc:23-36), elementwise ops
1e-4 (tests/test_cuda_ops.cc:20-21), attention 2e-3
(tests/test_cuda_attention.cc:23-24). Dequantisation, RoPE, embedding, KV
writes and argmax are compared bit for bit.
"""
import numpy as np
import pytest

import mini_llama_b200 as mlb
from mini_llama_b200 import configs as C

pytestmark = pytest.mark.gpu


def close(actual, expected, abs_tol, rel_tol=None):
    rel_tol = abs_tol if rel_tol is None else rel_tol
    actual, expected = np.asarray(actual, np.float64), np.asarray(expected, np.float64)
    err = np.abs(actual - expected)
    scale = np.maximum(1.0, np.abs(expected))
    ok = (err <= abs_tol) | (err / scale <= rel_tol)
    assert ok.all(), f"max err {err.max():.3e} at {np.unravel_index(err.argmax(), err.shape)}"


def pattern(shape, scale, shift, mult=19, add=7, mod=31):
    # MakePatternTensor, tests/test_cuda_quant.cc:52-60
    i = np.arange(int(np.prod(shape)))
    return ((((i * mult + add) % mod) - (mod // 2)) * scale + shift).astype(np.float32).reshape(shape)


def cpu_linear(port, qtype, x, blocks, n):
    """The reference CPU linear (oracle/_ref, all host threads) where built,
    else the C restatement (bit-identical, one thread)."""
    import os

    import oracle

    if oracle.ref_available():
        r = oracle.ref()
        r.set_threads(len(os.sched_getaffinity(0)))
        return r.linear(qtype, x, blocks, n)
    return port.linear(qtype, x, blocks, n)


def quantize(port, qtype, w):
    return port.quantize(qtype, w) if qtype != C.F32 else np.ascontiguousarray(w)


# ----------------------------------------------------------------- linear

@pytest.mark.parametrize("qtype", [C.Q8_0, C.Q4_0, C.Q4_1, C.F32])
def test_linear_reference_cases(cuda, port, qtype):
    torch = cuda
    cases = [((5, 13), (13,)), ((32, 64), (3, 64)), ((17, 65), (3, 65))]
    for wshape, xshape in cases:
        w = pattern(wshape, 0.037, -0.11)
        x = pattern(xshape, 0.071, 0.03)
        q = quantize(port, qtype, w)
        want = port.linear(qtype, x, q, wshape[0])
        xd = torch.from_numpy(x).cuda()
        wd = torch.from_numpy(q.view(np.uint8).reshape(-1)).cuda()
        nblk = wshape[0] * (wshape[1] if qtype == C.F32 else (wshape[1] + 31) // 32)
        fn = {C.Q8_0: mlb.CudaQ80LinearDeviceInput, C.Q4_0: mlb.CudaQ40LinearDeviceInput,
              C.Q4_1: mlb.CudaQ41LinearDeviceInput}.get(qtype)
        got = fn(xd, wd, nblk, wshape) if fn else mlb.CudaLinearDeviceInput(xd, wd, wshape)
        close(got.cpu().numpy(), want, 1e-3)
        bias = pattern((wshape[0],), 0.013, -0.02)
        host_fn = {C.Q8_0: mlb.CudaQ80Linear, C.Q4_0: mlb.CudaQ40Linear,
                   C.Q4_1: mlb.CudaQ41Linear}.get(qtype)
        got_h = host_fn(x, q, wshape, bias) if host_fn else mlb.CudaLinear(x, w, bias)
        close(got_h, want + bias, 1e-3)


def test_linear_rejects_bad_shapes(cuda):
    torch = cuda
    x = torch.zeros(64, device="cuda")
    w = torch.zeros(34 * 4, dtype=torch.uint8, device="cuda")
    with pytest.raises(mlb.MlbError, match="block count mismatch"):
        mlb.CudaQ80LinearDeviceInput(x, w, 3, [2, 64])
    with pytest.raises(mlb.MlbError, match="dimension mismatch"):
        mlb.CudaQ80LinearDeviceInput(x, w, 4, [2, 32])


SHAPES = [(4096, 4096), (1024, 4096), (11008, 4096), (4096, 11008), (515, 160), (100, 288),
          (8192, 29568 // 8 + 32)]


@pytest.mark.parametrize("qtype", [C.Q4_0, C.Q4_1, C.Q8_0])
@pytest.mark.parametrize("shape", SHAPES)
def test_qmatrix_gemv_vs_oracle(cuda, port, qtype, shape):
    torch = cuda
    n, k = shape
    blocks = C.synth_tensor(5, C.W_WQ, n % 97, qtype, n, k)
    qm = mlb.QMatrix.from_gguf(qtype, blocks, n, k)
    rng = np.random.default_rng(n + k)
    for rows in (1, 2, 4, 5):
        x = rng.normal(0, 1, (rows, k)).astype(np.float32)
        want = port.linear(qtype, x, blocks, n)
        got = qm.gemv(torch.from_numpy(x).cuda()).cpu().numpy()
        close(got, want, 1e-3)
        # deterministic: a second run is bit-identical
        again = qm.gemv(torch.from_numpy(x).cuda()).cpu().numpy()
        np.testing.assert_array_equal(got, again)


@pytest.mark.parametrize("qtype", [C.Q4_0, C.Q4_1, C.Q8_0])
@pytest.mark.parametrize("shape", [(4096, 4096), (11008, 4096), (1024, 4096), (515, 160),
                                   (300, 29568 // 8 + 32), (2048, 14336)])
def test_tensor_core_gemm_vs_oracle(cuda, port, qtype, shape):
    """The tcgen05 GEMM (batches: dequantised fp16 hi + lo weights in TMEM,
    fp16 hi + lo activations) against the reference CPU linear
    (LinearQ80/Q40/Q41, src/quant.cc:365-471) for batch widths 1..64 and a
    ragged 70-row batch (two passes), within the linear tolerance; reruns are
    bit-identical (split tiles are summed in chunk order)."""
    torch = cuda
    n, k = shape
    blocks = C.synth_tensor(5, C.W_WQ, n % 97, qtype, n, k)
    qm = mlb.QMatrix.from_gguf(qtype, blocks, n, k)
    rng = np.random.default_rng(n + 7 * k)
    for rows in (1, 5, 16, 17, 32, 48, 64, 70):
        x = rng.normal(0, 1, (rows, k)).astype(np.float32)
        want = cpu_linear(port, qtype, x, blocks, n).reshape(rows, n)
        xd = torch.from_numpy(x).cuda()
        got = qm.gemm(xd).cpu().numpy()
        close(got, want, 1e-3)
        np.testing.assert_array_equal(got, qm.gemm(xd).cpu().numpy())
        if rows > 4:  # the auto-routed entry point takes the same path
            np.testing.assert_array_equal(got, qm.gemv(xd).cpu().numpy())


def random_blocks(qtype, n, k, seed):
    """GGUF blocks with uniform random codes and random finite fp16 scales (and
    Q4_1 mins), subnormals and negative values included."""
    rng = np.random.default_rng(seed)
    nb, bs = (k + 31) // 32, C.BLOCK_BYTES[qtype]
    blk = rng.integers(0, 256, (n, nb, bs), dtype=np.uint8)
    nhalf = 2 if qtype == C.Q4_1 else 1
    h = rng.integers(0, 1 << 16, (n, nb, nhalf), dtype=np.uint32)
    h = np.where((h & 0x7C00) == 0x7C00, h & 0x83FF, h).astype(np.uint16)  # no inf/nan
    blk[:, :, :2 * nhalf] = h.view(np.uint8).reshape(n, nb, 2 * nhalf)
    return blk.reshape(n, nb * bs)


@pytest.mark.parametrize("qtype", [C.Q4_0, C.Q4_1, C.Q8_0])
@pytest.mark.parametrize("shape", [(4096, 4096), (11008, 4096), (14336, 4096), (515, 160),
                                   (100, 288), (33, 4128), (16, 32)])
def test_qmatrix_dequant_bit_exact(cuda, port, qtype, shape):
    """The repacked super-block layout decodes to exactly the reference's
    DequantizeFromQ80/Q40/Q41 (src/quant.cc:170-361): raw float32 bits equal,
    for the sweep shapes and ragged ones (K = 160, 288, 4128)."""
    import oracle

    n, k = shape
    blocks = random_blocks(qtype, n, k, n * 7 + k)
    qm = mlb.QMatrix.from_gguf(qtype, blocks, n, k)
    got = qm.dequant().cpu().numpy()
    want = port.dequant(qtype, blocks, n, k)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    if oracle.ref_available():
        ref = oracle.ref().dequant(qtype, blocks, n, k)
        np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
    # the same bits from a matrix the device generator filled (reference quantiser)
    dev = mlb.QMatrix.synthesize(qtype, n, k, 13, 4321)
    s = mlb._lib.synth_lib()
    nb = (k + 31) // 32
    hb = np.empty((n, nb * C.BLOCK_BYTES[qtype]), np.uint8)
    s.mlbs_gguf(qtype, s.mlbs_stream_key(13, 4321), 0.02, 0, 0, n, 0, nb, k, hb.ctypes.data,
                hb.shape[1], 8)
    np.testing.assert_array_equal(dev.dequant().cpu().numpy().view(np.uint32),
                                  port.dequant(qtype, hb, n, k).view(np.uint32))


def test_qmatrix_dequant_rejects_f32(cuda):
    w = np.ones((16, 32), np.float32)
    qm = mlb.QMatrix.from_gguf(C.F32, w, 16, 32)
    with pytest.raises(mlb.MlbError, match="F32"):
        qm.dequant()


@pytest.mark.parametrize("qtype", [C.Q4_0, C.Q4_1, C.Q8_0])
def test_device_generator_matches_host_generator(cuda, qtype):
    """Weights synthesised on the GPU equal the CPU generator's bytes: the
    GEMV of both is bit-identical."""
    torch = cuda
    n, k = 1000, 1056
    seed, sid = 9, 1234
    dev = mlb.QMatrix.synthesize(qtype, n, k, seed, sid)
    s = mlb._lib.synth_lib()
    key = s.mlbs_stream_key(seed, sid)
    nb = (k + 31) // 32
    host = np.empty((n, nb * C.BLOCK_BYTES[qtype]), np.uint8)
    s.mlbs_gguf(qtype, key, 0.02, 0, 0, n, 0, nb, k, host.ctypes.data, host.shape[1], 4)
    hm = mlb.QMatrix.from_gguf(qtype, host, n, k)
    x = torch.randn(1, k, device="cuda")
    np.testing.assert_array_equal(dev.gemv(x).cpu().numpy(), hm.gemv(x).cpu().numpy())


def test_qmatrix_raw_blocks_sweep_shape(cuda, port):
    torch = cuda
    for qtype in (C.Q4_0, C.Q4_1, C.Q8_0):
        n, k = 4096, 4096
        s = mlb._lib.synth_lib()
        key = s.mlbs_stream_key(3, 77)
        nb = k // 32
        host = np.empty((n, nb * C.BLOCK_BYTES[qtype]), np.uint8)
        s.mlbs_gguf(qtype, key, 0.0, 1, 0, n, 0, nb, k, host.ctypes.data, host.shape[1], 8)
        qm = mlb.QMatrix.from_gguf(qtype, host, n, k)
        dev = mlb.QMatrix.synthesize(qtype, n, k, 3, 77, raw=True)
        x = np.random.default_rng(1).normal(0, 1, (4, k)).astype(np.float32)
        want = port.linear(qtype, x, host, n)
        xd = torch.from_numpy(x).cuda()
        close(qm.gemv(xd).cpu().numpy(), want, 1e-3)
        np.testing.assert_array_equal(dev.gemv(xd).cpu().numpy(), qm.gemv(xd).cpu().numpy())


# -------------------------------------------------------------- elementwise

def test_elementwise_ops(cuda, port):
    torch = cuda
    for n in (32, 288, 4096, 8193):
        x = pattern((n,), 0.071, -0.13, 17, 5, 29)
        w = pattern((n,), 0.019, 1.0, 17, 5, 29)
        xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
        close(mlb.CudaRmsNormDeviceWeight(xd, wd, 1e-5).cpu().numpy(), port.rmsnorm(x, w, 1e-5), 1e-4)
        silu = x / (1.0 + np.exp(-x.astype(np.float64)))
        close(mlb.CudaSiluDeviceInput(xd).cpu().numpy(), silu, 1e-4)
        np.testing.assert_array_equal(mlb.CudaElementwiseMulDeviceInput(xd, wd).cpu().numpy(), x * w)
        np.testing.assert_array_equal(mlb.CudaElementwiseAddDeviceInput(xd, wd).cpu().numpy(), x + w)
        close(mlb.CudaSoftmax(xd).cpu().numpy(), port.softmax(x), 1e-4)


def test_embedding_and_argmax(cuda, port):
    torch = cuda
    table = C.synth_tensor(1, C.W_TOKEN_EMBEDDING, -1, C.F32, 1000, 96)
    td = torch.from_numpy(table).cuda()
    for tok in (0, 17, 999):
        np.testing.assert_array_equal(mlb.CudaEmbeddingLookupDeviceWeight(td, tok).cpu().numpy(),
                                      table[tok])
    with pytest.raises(mlb.MlbRangeError):
        mlb.CudaEmbeddingLookupDeviceWeight(td, 1000)
    rng = np.random.default_rng(0)
    for n in (1, 7, 32000, 152064):
        x = rng.normal(size=n).astype(np.float32)
        assert mlb.CudaArgMax(torch.from_numpy(x).cuda()) == port.argmax(x)
    tie = np.array([0.5, 3.0, 1.0, 3.0, 3.0], np.float32)
    assert mlb.CudaArgMax(torch.from_numpy(tie).cuda()) == 1


@pytest.mark.parametrize("neox", [0, 1])
def test_rope_bits(cuda, port, neox):
    torch = cuda
    rng = np.random.default_rng(neox)
    for heads, kv, d, theta in ((6, 6, 48, 10000.0), (32, 8, 128, 500000.0), (4, 1, 8, 1e6)):
        q = rng.normal(size=(heads, d)).astype(np.float32)
        k = rng.normal(size=(kv, d)).astype(np.float32)
        for pos in (0, 1, 255, 4095):
            qd, kd = torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda()
            mlb.CudaRopeDeviceInput(qd, kd, heads, kv, d, pos, theta, neox)
            wq, wk = port.rope(q, k, pos, theta, neox)
            np.testing.assert_array_equal(qd.cpu().numpy(), wq)
            np.testing.assert_array_equal(kd.cpu().numpy(), wk)


def test_kv_cache_write_and_bounds(cuda):
    torch = cuda
    cache = mlb.CudaKvCache(2, 8, 2, 4)
    k = torch.arange(8, dtype=torch.float32, device="cuda")
    v = -k
    cache.WriteDevice(1, 5, k, v)
    np.testing.assert_array_equal(cache.ReadKeyHead(1, 5, 1), [4, 5, 6, 7])
    np.testing.assert_array_equal(cache.ReadValueHead(1, 5, 0), [0, -1, -2, -3])
    assert not cache.keys[0].any()
    with pytest.raises(mlb.MlbRangeError):
        cache.WriteDevice(2, 0, k, v)
    with pytest.raises(mlb.MlbRangeError):
        cache.WriteDevice(0, 8, k, v)


# ----------------------------------------------------------------- attention

def test_attention_reference_direct_gqa(cuda, port):
    """tests/test_cuda_attention.cc:100-137 (pos = 1, head_dim = 3, GQA 2:1)."""
    torch = cuda
    q = np.array([0.2, -0.1, 0.4, -0.3, 0.5, 0.1], np.float32)
    keys = np.zeros((1, 4, 1, 3), np.float32)
    vals = np.zeros((1, 4, 1, 3), np.float32)
    keys[0, 0, 0], vals[0, 0, 0] = [0.1, 0.2, -0.1], [1.0, -2.0, 0.5]
    keys[0, 1, 0], vals[0, 1, 0] = [-0.4, 0.3, 0.2], [-1.0, 0.25, 2.0]
    cache = mlb.CudaKvCache(1, 4, 1, 3)
    cache.WriteDevice(0, 0, torch.from_numpy(keys[0, 0, 0]).cuda(), torch.from_numpy(vals[0, 0, 0]).cuda())
    cache.WriteDevice(0, 1, torch.from_numpy(keys[0, 1, 0]).cuda(), torch.from_numpy(vals[0, 1, 0]).cuda())
    want = port.attention(q.reshape(2, 3), keys, vals, 0, 1, 2, 1, 3, include_current_v=True)
    got = mlb.CudaAttentionDecodeDeviceInput(torch.from_numpy(q).cuda(), cache, 0, 1, 2, 1, 3)
    close(got.cpu().numpy().reshape(2, 3), want, 2e-3)


ATTN_CASES = [(6, 6, 48, 256), (8, 2, 32, 64), (32, 8, 128, 4096), (64, 8, 128, 1024),
              (32, 32, 128, 2048), (4, 1, 8, 40)]


@pytest.mark.parametrize("H,KV,D,S", ATTN_CASES)
@pytest.mark.parametrize("mode", [mlb.ATTN_STANDARD, mlb.ATTN_CPU_COMPAT])
def test_attention_vs_oracle(cuda, port, H, KV, D, S, mode):
    torch = cuda
    rng = np.random.default_rng(H * 7 + D)
    L = 2
    keys = rng.normal(0, 1, (L, S, KV, D)).astype(np.float32)
    vals = rng.normal(0, 1, (L, S, KV, D)).astype(np.float32)
    cache = mlb.CudaKvCache(L, S, KV, D)
    cache.keys.copy_(torch.from_numpy(keys))
    cache.values.copy_(torch.from_numpy(vals))
    for pos in sorted({0, 1, 31, 32, 33, S // 2, S - 1}):
        q = rng.normal(0, 1, (H, D)).astype(np.float32)
        want = port.attention(q, keys, vals, 1, pos, H, KV, D,
                              include_current_v=(mode == mlb.ATTN_STANDARD))
        got = mlb.CudaAttentionDecodeDeviceInput(torch.from_numpy(q).cuda(), cache, 1, pos, H, KV,
                                                 D, mode=mode)
        close(got.cpu().numpy().reshape(H, D), want, 2e-3)


def test_attention_bounds(cuda):
    torch = cuda
    cache = mlb.CudaKvCache(1, 4, 1, 8)
    q = torch.zeros(8, device="cuda")
    with pytest.raises(mlb.MlbRangeError):
        mlb.CudaAttentionDecodeDeviceInput(q, cache, 1, 0, 1, 1, 8)
    with pytest.raises(mlb.MlbRangeError):
        mlb.CudaAttentionDecodeDeviceInput(q, cache, 0, 4, 1, 1, 8)
