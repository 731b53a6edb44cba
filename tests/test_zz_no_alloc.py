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
