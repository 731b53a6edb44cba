"""Generates the golden fixtures in this directory from the reference itself.

Run in a checkout where the reference's CPU build exists (oracle/_ref/libmlref.so,
built by ``make -C oracle ref`` from the reference sources):

    python tests/golden/make_golden.py

Every number here comes from the reference's own code (ForwardToken with no CUDA
weights, ArgMax) fed with seeded synthetic weights from
mini_llama_b200.configs (or, for ``tiny_readme``, the reference's own fixture
model models/tiny/model.{json,bin}). The fixtures pin the C restatement in
oracle/port and are the parity targets of the GPU tests.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from mini_llama_b200 import configs as C  # noqa: E402

# the reference checkout: $REF_ROOT, else the one named `reference` beside this repository
REF_ROOT = os.environ.get("REF_ROOT") or os.path.join(os.path.dirname(ROOT), "reference")

# Small models covering the code paths (GQA, NeoX + bias, ragged shapes).
SMALL = {
    "small_q4_0_gqa": (dict(vocab_size=1000, dim=256, hidden_dim=512, n_layers=2, n_heads=8,
                            n_kv_heads=2, head_dim=32, max_seq_len=64, rope_theta=10000.0,
                            rms_norm_eps=1e-5, rope_type=0), C.Q4_0, False),
    "small_q4_1_neox_bias": (dict(vocab_size=1000, dim=256, hidden_dim=384, n_layers=2,
                                  n_heads=4, n_kv_heads=2, head_dim=64, max_seq_len=64,
                                  rope_theta=1000000.0, rms_norm_eps=1e-6, rope_type=1),
                             C.Q4_1, True),
    "small_q8_0_ragged": (dict(vocab_size=515, dim=160, hidden_dim=224, n_layers=2, n_heads=5,
                               n_kv_heads=1, head_dim=32, max_seq_len=48, rope_theta=10000.0,
                               rms_norm_eps=1e-5, rope_type=0), C.Q8_0, False),
}
SMALL_PROMPT, SMALL_STEPS = 8, 24
TINY_SEED, TINY_PROMPT, TINY_STEPS = 1, 16, 128
TINY_LOGIT_STEPS = [0, 15, 16, 143]


def weights_digest(weights) -> str:
    h = hashlib.sha256()
    for kind, layer, qtype, rows, cols, arr in weights:
        h.update(np.array([kind, layer, qtype, rows, cols], np.int64).tobytes())
        h.update(np.ascontiguousarray(arr).tobytes())
    return h.hexdigest()


def run_greedy(model, prompt, steps):
    """Prefill the prompt, then `steps` greedy tokens; returns per-step logits."""
    logits, tokens = [], []
    tok = prompt[0]
    for pos in range(len(prompt) + steps):
        lg = model.forward_token(tok, pos)
        logits.append(lg)
        nxt = int(np.argmax(lg))  # same rule as ArgMax: first maximal index
        tokens.append(nxt)
        tok = prompt[pos + 1] if pos + 1 < len(prompt) else nxt
    return np.stack(logits), tokens


def top2_margin(lg):
    s = np.sort(lg)
    return float(s[-1] - s[-2])


def make_model(ref, cfg, qtype, seed, bias):
    m = ref.model(cfg)
    ws = list(C.host_weights(cfg, qtype, seed, bias))
    for kind, layer, qt, rows, cols, arr in ws:
        m.set_weight(kind, layer, qt, rows, cols, arr)
    return m, weights_digest(ws)


def main():
    ref = oracle.ref()
    ref.set_threads(os.cpu_count() or 8)
    meta = {}

    # 1. The reference's own tiny fixture model (models/tiny/model.{json,bin}: a
    #    manifest of float32 tensors at byte offsets) and README prompt "hello".
    with open(os.path.join(REF_ROOT, "models/tiny/model.json")) as f:
        manifest = json.load(f)
    blob = np.fromfile(os.path.join(REF_ROOT, "models/tiny/model.bin"), dtype=np.uint8)
    mc = manifest["config"]
    cfg = dict(vocab_size=mc["vocab_size"], dim=mc["dim"], hidden_dim=mc["hidden_dim"],
               n_layers=mc["n_layers"], n_heads=mc["n_heads"], n_kv_heads=mc["n_kv_heads"],
               head_dim=mc["dim"] // mc["n_heads"], max_seq_len=mc["max_seq_len"],
               rope_theta=float(mc["rope_theta"]), rms_norm_eps=float(mc["rms_norm_eps"]),
               rope_type=0)
    names = {"token_embedding": (0, -1), "final_norm": (1, -1), "lm_head": (2, -1)}
    for layer in range(cfg["n_layers"]):
        for kind, nm in ((3, "attention_norm"), (4, "wq"), (5, "wk"), (6, "wv"), (10, "wo"),
                         (11, "ffn_norm"), (12, "w_gate"), (13, "w_up"), (14, "w_down")):
            names[f"layers.{layer}.{nm}"] = (kind, layer)
    arrays = {}
    rm = ref.model(cfg)
    for t in manifest["tensors"]:
        if t["name"] not in names:
            continue
        kind, layer = names[t["name"]]
        arr = blob[t["offset"]:t["offset"] + t["byte_size"]].view(np.float32).copy()
        rows, cols = C.weight_shape(cfg, kind)
        arr = arr.reshape(rows, cols)
        arrays[f"w{kind}" + ("" if layer < 0 else f"_{layer}")] = arr
        rm.set_weight(kind, layer, C.F32, rows, cols, arr)
    prompt = [1, 104, 101, 108, 108, 111]  # README.md:287 ("hello")
    logits, toks = run_greedy(rm, prompt, 64)
    np.savez_compressed(os.path.join(HERE, "tiny_readme.npz"), logits=logits,
                        tokens=np.array(toks, np.int32), prompt=np.array(prompt, np.int32),
                        **arrays)
    meta["tiny_readme"] = dict(config=cfg, prompt=prompt, generated=toks[len(prompt) - 1:],
                               note="weights are the reference's models/tiny fixture")

    # 2. BASELINE tiny config, Q8_0, 16 prompt ids + 128 greedy steps.
    m, digest = make_model(ref, C.TINY, C.Q8_0, TINY_SEED, False)
    prompt = C.prompt_ids(TINY_SEED, TINY_PROMPT, C.TINY["vocab_size"])
    logits, toks = run_greedy(m, prompt, TINY_STEPS)
    np.savez_compressed(os.path.join(HERE, "tiny_q8_0.npz"),
                        logits=logits[TINY_LOGIT_STEPS], logit_steps=np.array(TINY_LOGIT_STEPS),
                        tokens=np.array(toks, np.int32), prompt=np.array(prompt, np.int32),
                        margins=np.array([top2_margin(l) for l in logits], np.float32))
    meta["tiny_q8_0"] = dict(config=C.TINY, qtype="q8_0", seed=TINY_SEED, prompt=prompt,
                             weights_sha256=digest, generated=toks[TINY_PROMPT - 1:])

    # 3. Small models with every code path.
    for name, (cfg, qtype, bias) in SMALL.items():
        m, digest = make_model(ref, cfg, qtype, 7, bias)
        prompt = C.prompt_ids(7, SMALL_PROMPT, cfg["vocab_size"])
        logits, toks = run_greedy(m, prompt, SMALL_STEPS)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), logits=logits,
                            tokens=np.array(toks, np.int32), prompt=np.array(prompt, np.int32))
        meta[name] = dict(config=cfg, qtype=C.QTYPE_NAMES[qtype], seed=7, bias=bias,
                          prompt=prompt, weights_sha256=digest)

    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print(json.dumps({k: v.get("generated", "")[:12] for k, v in meta.items()}))


if __name__ == "__main__":
    main()
