"""Tensor-parallel plan on the host (no GPU).

* Coverage: for every bench workload and TP size the shards tile the query
  heads, KV heads (with the GQA map kept inside each rank), FFN hidden rows
  (whole 32-row blocks, as even as the blocks allow) and the vocabulary.
* Collectives: two gloo ranks run one decode layer sharded exactly as the
  plan says (numpy arithmetic, torch.distributed all-reduce / all-gather), and
  the vocab-sharded lm_head's packed argmax keys reduced with MAX; rank 0
  checks the result against the unsharded layer and the global argmax (ties
  to the lowest index, as ArgMax, src/ops.cc:220-233).
"""
import socket

import numpy as np
import pytest

import mini_llama_b200 as mlb
from mini_llama_b200 import configs as C


def shards(cfg, tp):
    return [mlb.tp_plan(cfg, r, tp) for r in range(tp)]


@pytest.mark.parametrize("name", ["llama2-7b-q4_0", "llama3-8b-q8_0", "qwen2-72b-q4_1"])
@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_shards_tile_every_dimension(name, tp):
    cfg = C.WORKLOADS[name][0]
    sh = shards(cfg, tp)
    gq = cfg["n_heads"] // cfg["n_kv_heads"]
    for field, total in (("q_head", cfg["n_heads"]), ("kv_head", cfg["n_kv_heads"]),
                         ("ffn_row", cfg["hidden_dim"]), ("vocab_row", cfg["vocab_size"])):
        count = field + "s"
        start = 0
        for s in sh:
            assert s[field + "0"] == start, (field, s)
            start += s[count]
        assert start == total, field
    for s in sh:
        assert s["q_heads"] == s["kv_heads"] * gq          # whole GQA groups per rank
        assert s["q_head0"] == s["kv_head0"] * gq
        assert s["ffn_row0"] % 32 == 0 and s["ffn_rows"] % 32 == 0
    rows = [s["ffn_rows"] for s in sh]
    assert max(rows) - min(rows) <= 32                      # blocks split evenly


def test_unsplittable_configs_are_rejected():
    with pytest.raises(mlb.MlbError, match="divisible by the TP size"):
        mlb.tp_plan(C.TINY, 0, 4)          # 6 heads over 4 ranks
    with pytest.raises(mlb.MlbError, match="multiple of 32"):
        mlb.tp_plan(C.TINY, 0, 2)          # 3 heads x 48 = 144 columns per rank
    with pytest.raises(mlb.MlbError, match="bad tensor-parallel rank"):
        mlb.tp_plan(C.LLAMA2_7B, 2, 2)


# ------------------------------------------------------------ gloo ranks

LAYER = dict(vocab_size=10, dim=64, hidden_dim=96, n_layers=1, n_heads=4, n_kv_heads=2,
             head_dim=16, max_seq_len=16, rope_theta=10000.0, rms_norm_eps=1e-5, rope_type=0)


def rmsnorm(x, w, eps):
    return x / np.sqrt(np.mean(x * x) + eps) * w


def layer_weights(cfg, seed=3):
    rng = np.random.default_rng(seed)
    D, H, KV, F, V = cfg["head_dim"], cfg["n_heads"], cfg["n_kv_heads"], cfg["hidden_dim"], \
        cfg["vocab_size"]
    d = cfg["dim"]
    w = {k: rng.normal(0, 0.1, shape) for k, shape in (
        ("wq", (H * D, d)), ("wk", (KV * D, d)), ("wv", (KV * D, d)), ("wo", (d, H * D)),
        ("wg", (F, d)), ("wu", (F, d)), ("wd", (d, F)), ("lm", (V, d)))}
    w["n1"] = rng.normal(1, 0.1, d)
    w["n2"] = rng.normal(1, 0.1, d)
    w["nf"] = rng.normal(1, 0.1, d)
    w["x"] = rng.normal(0, 1, d)
    T = 5  # cached positions, the last one is the current token's
    w["kc"] = rng.normal(0, 1, (T, KV * D))
    w["vc"] = rng.normal(0, 1, (T, KV * D))
    # the greedy token tied across the two vocabulary shards (rows 2 and 7 point
    # along the final normalised hidden state, so they hold the maximum)
    xo, _ = full_layer(cfg, w)
    xf = rmsnorm(xo, w["nf"], cfg["rms_norm_eps"])
    w["lm"][2] = w["lm"][7] = 3.0 * xf / np.linalg.norm(xf)
    return w


def attention(q, kc, vc, H, KV, D):
    gq = H // KV
    out = np.zeros(H * D)
    for h in range(H):
        kvh = h // gq
        s = kc[:, kvh * D:(kvh + 1) * D] @ q[h * D:(h + 1) * D] / np.sqrt(D)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h * D:(h + 1) * D] = p @ vc[:, kvh * D:(kvh + 1) * D]
    return out


def silu(g):
    return g / (1 + np.exp(-g))


def full_layer(cfg, w):
    eps, D, H, KV = cfg["rms_norm_eps"], cfg["head_dim"], cfg["n_heads"], cfg["n_kv_heads"]
    xn = rmsnorm(w["x"], w["n1"], eps)
    q = w["wq"] @ xn
    xb = w["x"] + w["wo"] @ attention(q, w["kc"], w["vc"], H, KV, D)
    xbn = rmsnorm(xb, w["n2"], eps)
    xo = xb + w["wd"] @ (silu(w["wg"] @ xbn) * (w["wu"] @ xbn))
    return xo, w["lm"] @ rmsnorm(xo, w["nf"], eps)


def argmax_key(v, index):
    """The device's packed greedy key (argmax_key_of): order-preserving float32
    bits << 32 | (2^32 - 1 - index), mapped to signed int64 order."""
    u = int(np.float32(v).view(np.uint32))
    u = (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)
    key = (u << 32) | (0xFFFFFFFF - index)
    return key - (1 << 63)  # unsigned order -> signed order


def rank_main(rank, world, port, out):
    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        cfg = LAYER
        sh = mlb.tp_plan(cfg, rank, world)
        w = layer_weights(cfg)
        eps, D = cfg["rms_norm_eps"], cfg["head_dim"]
        qr = slice(sh["q_head0"] * D, (sh["q_head0"] + sh["q_heads"]) * D)
        kvr = slice(sh["kv_head0"] * D, (sh["kv_head0"] + sh["kv_heads"]) * D)
        fr = slice(sh["ffn_row0"], sh["ffn_row0"] + sh["ffn_rows"])
        vr = slice(sh["vocab_row0"], sh["vocab_row0"] + sh["vocab_rows"])

        def allreduce(v):
            t = torch.from_numpy(np.ascontiguousarray(v))
            dist.all_reduce(t)
            return t.numpy()

        xn = rmsnorm(w["x"], w["n1"], eps)
        q = w["wq"][qr] @ xn                                   # column-sharded wq
        att = attention(q, w["kc"][:, kvr], w["vc"][:, kvr], sh["q_heads"], sh["kv_heads"], D)
        xb = w["x"] + allreduce(w["wo"][:, qr] @ att)          # row-sharded wo + all-reduce
        xbn = rmsnorm(xb, w["n2"], eps)
        h = silu(w["wg"][fr] @ xbn) * (w["wu"][fr] @ xbn)      # column-sharded gate/up
        xo = xb + allreduce(w["wd"][:, fr] @ h)                # row-sharded down + all-reduce
        lg = (w["lm"][vr] @ rmsnorm(xo, w["nf"], eps)).astype(np.float32)
        keys = [argmax_key(v, sh["vocab_row0"] + i) for i, v in enumerate(lg)]
        key = torch.tensor([max(keys)], dtype=torch.int64)
        dist.all_reduce(key, op=dist.ReduceOp.MAX)             # greedy token across shards
        gathered = [torch.zeros(sh["vocab_rows"], dtype=torch.float32) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(lg))
        if rank == 0:
            k = int(key.item()) + (1 << 63)
            np.savez(out, xo=xo, logits=torch.cat(gathered).numpy(),
                     token=0xFFFFFFFF - (k & 0xFFFFFFFF))
    finally:
        dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_match_the_unsharded_layer(tmp_path):
    import torch.multiprocessing as mp

    out = str(tmp_path / "tp.npz")
    sh = shards(LAYER, 2)
    assert [s["ffn_rows"] for s in sh] == [32, 64]  # an uneven FFN split is exercised
    mp.start_processes(rank_main, args=(2, free_port(), out), nprocs=2, join=True,
                       start_method="spawn")
    got = np.load(out)
    xo, logits = full_layer(LAYER, layer_weights(LAYER))
    np.testing.assert_allclose(got["xo"], xo, rtol=0, atol=1e-12)
    np.testing.assert_allclose(got["logits"], logits.astype(np.float32), rtol=1e-6, atol=1e-6)
    lg32 = logits.astype(np.float32)
    assert lg32[2] == lg32[7] == lg32.max()          # tied across the two shards
    assert int(got["token"]) == 2                    # lowest index wins


# ------------------------------------------------- a rank that fails (host side)

def failing_rank_main(rank, world, port, out_dir):
    """Rank 1 raises before the all-reduce that exchanges per-rank step times
    (bench.py's max over ranks); rank 0 must see an error from its collective
    within the process group's timeout and record it, not wait for ever."""
    import datetime
    import os
    import time

    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    t0 = time.perf_counter()
    try:
        t = torch.tensor([1.0])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        outcome = "completed"
    except Exception as e:  # the failure surfaces as an error on the survivor
        outcome = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(f"{outcome}\n{time.perf_counter() - t0:.2f}\n")


def test_failed_rank_surfaces_as_an_error(tmp_path):
    import torch.multiprocessing as mp

    ctx = mp.start_processes(failing_rank_main, args=(2, free_port(), str(tmp_path)), nprocs=2,
                             join=False, start_method="spawn")
    for p in ctx.processes:  # each ends by itself: rank 1 raises, rank 0 times out or errors
        p.join(timeout=120)
    alive = [p for p in ctx.processes if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank did not end after its peer failed"
    assert ctx.processes[1].exitcode != 0          # the injected failure
    assert ctx.processes[0].exitcode == 0          # the survivor handled it
    outcome, secs = (tmp_path / "rank0.txt").read_text().split("\n")[:2]
    assert outcome.startswith("error"), outcome     # its collective failed ...
    assert float(secs) < 30.0                       # ... within the process-group timeout
