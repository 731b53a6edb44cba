"""Failure detection on the GPU without a fault: each bounded wait of the
decode-step kernel (the weight ring's mbarrier wait, the grid barrier) is
made to wait for something that never comes, with a 1 ms limit, through the
C ABI (mlb_wait_selftest). The wait must give up, report MLB_ERR_TIMEOUT and
its site in the status word, and leave the GPU usable: a GEMV right after
still matches the oracle."""
import time

import numpy as np
import pytest

import mini_llama_b200 as mlb
from mini_llama_b200 import configs as C

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("which", [0, 1])
def test_bounded_wait_gives_up_and_reports(cuda, port, which):
    torch = cuda
    t0 = time.perf_counter()
    code, where = mlb.wait_selftest(which, limit_ms=1.0)
    elapsed = time.perf_counter() - t0
    assert code == mlb.ERR_TIMEOUT
    assert where == 900 + which
    assert elapsed < 1.5  # gave up after its 1 ms limit, not the production ~2 s
    # the GPU is still usable: a quantised GEMV against the oracle
    n, k = 64, 512
    blocks = C.synth_tensor(7, C.W_WQ, 3, C.Q4_0, n, k)
    qm = mlb.QMatrix.from_gguf(C.Q4_0, blocks, n, k)
    x = np.random.default_rng(1).normal(0, 1, (1, k)).astype(np.float32)
    got = qm.gemv(torch.from_numpy(x).cuda()).cpu().numpy()
    want = port.linear(C.Q4_0, x, blocks, n)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-3 * max(1.0, np.abs(want).max()))


def test_selftest_rejects_bad_arguments(cuda):
    with pytest.raises(mlb.MlbError, match="which must be 0 or 1"):
        mlb.wait_selftest(2)
    with pytest.raises(mlb.MlbError, match="limit_ms"):
        mlb.wait_selftest(0, limit_ms=0.0)
