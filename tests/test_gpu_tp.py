"""Tensor-parallel decode on 2 GPUs (skipped with fewer): the golden small
models sharded over two ranks, on both step paths (the persistent kernel with
its partial sums exchanged over NVLink peer memory, and the per-op graph with
NCCL all-reduce after wo and w_down), vocab-sharded lm_head with the greedy
key reduced by MAX, against the reference CPU path's golden logits and token
ids."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LOGIT_TOL = 2e-3


def gpus():
    torch = pytest.importorskip("torch")
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("path", ["step", "per_op"])
@pytest.mark.parametrize("name", ["small_q4_0_gqa", "small_q4_1_neox_bias"])
def test_two_rank_decode_matches_reference(name, path, tmp_path):
    if gpus() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "tp.json"
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(free_port()), os.path.join(ROOT, "tests", "tp_worker.py"),
           name, str(out), path]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    res = json.loads(out.read_text())
    assert res["step_kernel"] == (path == "step")
    assert res["max_err"] <= LOGIT_TOL
    n = res["prompt_len"]
    assert res["argmax"] == res["gold"]                    # teacher-forced: same inputs
    assert res["device_greedy"] == res["gold"][n - 1:]     # free-running on the device


@pytest.mark.parametrize("path", ["step", "per_op", "batch"])
@pytest.mark.parametrize("model", ["synth7b", "synth72b"])
def test_tp_greedy_ids_match_one_gpu(model, path, tmp_path):
    """Every available rank count (2, 4, 8): a 7B-shaped model (4 layers) and a
    Qwen2-72B-shaped one (2 layers: Q4_1, bias, NeoX, GQA 8) decoded greedily
    at TP=N give the single-GPU ids; logits within the bar. "batch": 8
    sequences through the batched engine (tensor-core GEMMs)."""
    n = gpus()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    world = 8 if n >= 8 else (4 if n >= 4 else 2)
    out = tmp_path / "tp.json"
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", str(world), "--master-addr", "127.0.0.1",
           "--master-port", str(free_port()), os.path.join(ROOT, "tests", "tp_worker.py"),
           model, str(out), path]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    res = json.loads(out.read_text())
    assert res["step_kernel"] == (path == "step")
    assert res["tp_ids"] == res["ids"]
    assert res["max_err"] <= LOGIT_TOL
