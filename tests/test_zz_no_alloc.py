"""mlb_attention_decode_noalloc: decode attention for callers that cannot
allocate device memory during the call (a host whose device memory belongs to
its own fixed-budget allocator, or a latency-critical loop that cannot take
cudaMalloc/cudaFree's synchronisation). It keeps its split-K scratch in a fixed
array inside the library instead of allocating it.

Checked through the C ABI against the allocating entry point
mlb_attention_decode, on two calls in a row (the second call finds the
scratch, including the arrival counters, as the first left it), within the
attention tolerance of the reference's GPU tests (2e-3,
tests/test_cuda_attention.cc:23-24). Collected last on purpose.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _attention(lib, fn, q, keys, values, layer, pos, H, KV, D, mode):
    import torch

    L, S = keys.shape[0], keys.shape[1]
    out = torch.empty(H * D, dtype=torch.float32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = getattr(lib, fn)(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(keys.data_ptr()),
                          ctypes.c_void_p(values.data_ptr()), L, S, layer, pos, H, KV, D, mode,
                          ctypes.c_void_p(out.data_ptr()), 0, stream)
    assert rc == 0, lib.mlb_last_error().decode()
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("H,KV,D,S", [(32, 8, 128, 2048), (32, 32, 128, 1024), (4, 1, 12, 40)])
@pytest.mark.parametrize("mode", [0, 1])
def test_noalloc_matches_allocating_entry_point(H, KV, D, S, mode):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mini_llama_b200 import _lib

    lib = _lib.lib()
    gen = torch.Generator(device="cuda").manual_seed(H * 1000 + D + mode)
    keys = torch.randn(2, S, KV, D, device="cuda", generator=gen)
    values = torch.randn(2, S, KV, D, device="cuda", generator=gen)
    for call, pos in enumerate((S - 1, S // 3)):  # two calls in a row
        q = torch.randn(H * D, device="cuda", generator=gen)
        want = _attention(lib, "mlb_attention_decode", q, keys, values, 1, pos, H, KV, D, mode)
        got = _attention(lib, "mlb_attention_decode_noalloc", q, keys, values, 1, pos, H, KV, D,
                         mode)
        err = np.abs(got - want) / np.maximum(1.0, np.abs(want))
        assert err.max() <= TOL, f"call {call}: max error {err.max():.2e}"


@pytest.mark.parametrize("H,KV,D,S", [
    (2048, 128, 128, 256),  # one split needs 266,240 floats: 3 splits fit where 4 are wanted
    (32, 8, 128, 300),      # GQA 4:1, the 8B shape
    (4, 2, 10, 40),         # head_dim not a multiple of 4: the generic kernel (no scratch)
])
def test_noalloc_matches_oracle(port, H, KV, D, S):
    """Against the CPU oracle (oracle/port, the reference CPU attention with
    its V-sum rule, src/forward.cc:463-545), not only against the allocating
    entry point: a shape whose split count is cut to fit the fixed scratch, a
    GQA shape, and a head_dim that takes the generic kernel. Two calls each."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mini_llama_b200 import _lib

    lib = _lib.lib()
    gen = torch.Generator(device="cuda").manual_seed(H + KV + D)
    keys = torch.randn(2, S, KV, D, device="cuda", generator=gen)
    values = torch.randn(2, S, KV, D, device="cuda", generator=gen)
    kn, vn = keys.cpu().numpy(), values.cpu().numpy()
    for mode in (0, 1):
        for pos in (S - 1, S // 2):
            q = torch.randn(H * D, device="cuda", generator=gen)
            got = _attention(lib, "mlb_attention_decode_noalloc", q, keys, values, 1, pos, H, KV,
                             D, mode)
            want = port.attention(q.cpu().numpy(), kn, vn, 1, pos, H, KV, D,
                                  include_current_v=bool(mode)).reshape(-1)
            err = np.abs(got - want) / np.maximum(1.0, np.abs(want))
            assert err.max() <= TOL, f"mode {mode} pos {pos}: max error {err.max():.2e}"
            alloc = _attention(lib, "mlb_attention_decode", q, keys, values, 1, pos, H, KV, D,
                               mode)
            err = np.abs(got - alloc) / np.maximum(1.0, np.abs(alloc))
            assert err.max() <= TOL


def test_noalloc_rejects_a_split_beyond_its_scratch():
    """KV = 256, 16 query heads per KV head, head_dim 256: one split alone needs
    256 * 16 * 258 = 1,056,768 partial floats, above the 2^20 the array holds."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mini_llama_b200 import _lib

    lib = _lib.lib()
    buf = torch.zeros(16, device="cuda")
    p = ctypes.c_void_p(buf.data_ptr())
    rc = lib.mlb_attention_decode_noalloc(p, p, p, 1, 4, 0, 1, 4096, 256, 256, 0, p, 0, None)
    assert rc == -1
    assert b"scratch floats, above the fixed limit of 1048576" in lib.mlb_last_error()


def test_noalloc_rejects_shapes_beyond_its_scratch():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mini_llama_b200 import _lib

    lib = _lib.lib()
    keys = torch.zeros(1, 4, 2048, 4, device="cuda")
    q = torch.zeros(2048 * 4, device="cuda")
    out = torch.zeros(2048 * 4, device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    rc = lib.mlb_attention_decode_noalloc(p(q), p(keys), p(keys), 1, 4, 0, 1, 2048, 2048, 4, 1,
                                          p(out), 0, None)
    assert rc == -1
    assert b"exceeds the fixed scratch limit" in lib.mlb_last_error()
