"""One rank of a tensor-parallel decode run (launched by torch.distributed.run,
one process per GPU) for tests/test_gpu_tp.py: loads a golden small model
sharded over WORLD_SIZE ranks and decodes it with the step path named on the
command line ("step": the persistent kernel exchanging partial sums over
NVLink peer memory; "per_op": one kernel per op with NCCL); rank 0 writes the
logits and token ids to the JSON file named on the command line."""
import datetime
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import mini_llama_b200 as mlb  # noqa: E402
from mini_llama_b200 import configs as C  # noqa: E402


# Full-width shapes cut to a few layers, seeded on the device so every rank and
# the single-GPU copy hold the same weights: (config, format, q/k/v bias).
SYNTH = {
    "synth7b": (dict(C.LLAMA2_7B, n_layers=4), C.Q4_0, False),
    # Qwen2-72B width: NeoX RoPE, q/k/v bias, GQA 64/8, hidden 29568 (not a
    # multiple of 256 per rank)
    "synth72b": (dict(C.QWEN2_72B, n_layers=2), C.Q4_1, True),
}


def synth_vs_single(name, out, step_kernel, rank, world, local, nccl_id):
    """Greedy ids of a SYNTH model at TP=world against one GPU."""
    base, qt, bias = SYNTH[name]
    cfg = dict(base, max_seq_len=256)
    steps = 48
    model = mlb.CudaModel(cfg, device_id=local, tp_rank=rank, tp_size=world, nccl_id=nccl_id)
    model.synthesize(qt, 77, with_bias=bias)
    ctx = model.context(step_kernel=step_kernel)
    tp_ids = ctx.decode_greedy(11, 0, steps)
    lg = ctx.forward_token(tp_ids[-1], steps)
    used = ctx.step_kernel()
    ctx.close()
    model.close()
    dist.barrier()
    if rank == 0:
        one = mlb.CudaModel(cfg, device_id=local).synthesize(qt, 77, with_bias=bias)
        c1 = one.context()
        ids = c1.decode_greedy(11, 0, steps)
        l1 = c1.forward_token(ids[-1], steps)
        with open(out, "w") as f:
            json.dump({"tp_ids": tp_ids, "ids": ids, "step_kernel": used,
                       "max_err": float(np.abs(lg - l1).max())}, f)
        c1.close()
        one.close()
    dist.barrier()


def synth_batch_vs_single(name, out, rank, world, local, nccl_id):
    """The batched engine at TP=world (tensor-core GEMMs on each rank's shard,
    NCCL all-reduce after wo and w_down, vocab-sharded greedy keys) against one
    GPU: 8 sequences of different seeded K/V lengths decoded in lockstep."""
    base, qt, bias = SYNTH[name]
    cfg = dict(base, max_seq_len=512)
    n_seqs, steps = 8, 12
    starts = [40 + 37 * s for s in range(n_seqs)]
    toks = [11 + 101 * s for s in range(n_seqs)]

    def run(model):
        b = mlb.Batch(model, n_seqs)
        for s in range(n_seqs):
            b.fill_kv(s, starts[s], 5 + s)
        ids = b.decode_greedy(toks, starts, steps)
        _, lg = b.forward(list(range(n_seqs)), ids[-1], [p + steps for p in starts], logits=True)
        b.close()
        return ids, lg

    model = mlb.CudaModel(cfg, device_id=local, tp_rank=rank, tp_size=world, nccl_id=nccl_id)
    model.synthesize(qt, 77, with_bias=bias)
    tp_ids, tp_lg = run(model)
    model.close()
    dist.barrier()
    if rank == 0:
        one = mlb.CudaModel(cfg, device_id=local).synthesize(qt, 77, with_bias=bias)
        ids, lg = run(one)
        one.close()
        with open(out, "w") as f:
            json.dump({"tp_ids": tp_ids.tolist(), "ids": ids.tolist(), "step_kernel": False,
                       "max_err": float(np.abs(tp_lg - lg).max())}, f)
    dist.barrier()


def main():
    name, out, path = sys.argv[1], sys.argv[2], sys.argv[3]
    step_kernel = path == "step"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    obj = [mlb.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    if name in SYNTH and path == "batch":
        synth_batch_vs_single(name, out, rank, world, local, obj[0])
        dist.destroy_process_group()
        return
    if name in SYNTH:
        synth_vs_single(name, out, step_kernel, rank, world, local, obj[0])
        dist.destroy_process_group()
        return
    golden = os.path.join(ROOT, "tests", "golden")
    with open(os.path.join(golden, "golden.json")) as f:
        mt = json.load(f)[name]
    g = np.load(os.path.join(golden, f"{name}.npz"))
    qtype = {v: k for k, v in C.QTYPE_NAMES.items()}[mt["qtype"]]
    cfg = mt["config"]
    model = mlb.CudaModel(cfg, device_id=local, tp_rank=rank, tp_size=world, nccl_id=obj[0])
    model.load(list(C.host_weights(cfg, qtype, mt["seed"], mt["bias"])))
    prompt = [int(t) for t in g["prompt"]]
    gold = [int(t) for t in g["tokens"]]
    # teacher-forced logits (every rank runs the same steps: the step holds collectives)
    ctx = model.context(step_kernel=step_kernel)
    logits, tok = [], prompt[0]
    for pos in range(len(gold)):
        logits.append(ctx.forward_token(tok, pos))
        tok = prompt[pos + 1] if pos + 1 < len(prompt) else gold[pos]
    # the on-device greedy loop
    ctx2 = model.context(step_kernel=step_kernel)
    for pos, t in enumerate(prompt[:-1]):
        ctx2.forward_token(t, pos)
    dev = ctx2.decode_greedy(prompt[-1], len(prompt) - 1, len(gold) - len(prompt) + 1)
    if rank == 0:
        err = np.abs(np.stack(logits) - g["logits"]).max()
        with open(out, "w") as f:
            json.dump({"max_err": float(err), "argmax": [int(np.argmax(l)) for l in logits],
                       "device_greedy": dev, "gold": gold, "prompt_len": len(prompt),
                       "kernels_per_step": ctx.kernels_per_step(),
                       "step_kernel": ctx.step_kernel()}, f)
    ctx.close()
    ctx2.close()
    model.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
