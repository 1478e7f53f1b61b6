"""Generates the golden decode fixtures in this directory from the REFERENCE's
own C++ port (oracle/_ref/refdrv*, compiled from the reference sources by
oracle/Makefile).  Run in the build container, where the reference exists:

    python tests/golden/make_golden.py [case ...] [--workers N]

Each fixture pins, per sequence, the final witness digest (CIS2_REF /
CIS2_SAMPLE digest), the argmax digest, and `steps_sha` = SHA-256 over the
concatenated 32-byte per-step witness digests; the first sequence also keeps
its full token stream and every per-step digest.  Inputs are regenerated
from seeds by cis2-lab-archive_b200/synth.py, so the fixtures stay small.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
synth = importlib.import_module("cis2-lab-archive_b200.synth")
import pyoracle  # noqa: E402

SAMPLE = {"seed": 20261201, "temperature": 0.8, "top_p": 0.95}

# name -> (model, prompts spec, gen, tree, sampled)
#   prompts spec: ("workload", name, first, count), ("workload_idx", name, [sequence indices])
#   or ("random", seed, [lens])
CASES = {
    "tiny_seq_greedy": ("tiny", ("random", 11, [1, 5, 9, 16]), 12, False, False),
    "tiny_tree_greedy": ("tiny", ("random", 11, [1, 5, 9, 16]), 12, True, False),
    "tiny_seq_sampled": ("tiny", ("random", 12, [3, 7]), 12, False, True),
    "tiny_tree_sampled": ("tiny", ("random", 12, [3, 7]), 12, True, True),
    "tiny_mha_untied_seq": ("tiny_mha_untied", ("random", 13, [2, 33, 40]), 16, False, False),
    "tiny_mha_untied_tree": ("tiny_mha_untied", ("random", 13, [2, 33, 40]), 16, True, False),
    "tiny_qwen3_seq_greedy": ("tiny_qwen3", ("random", 14, [4, 6]), 12, False, False),
    "tiny_qwen3_seq_sampled": ("tiny_qwen3", ("random", 14, [4, 6]), 12, False, True),
    "tiny_qwen3_tree_sampled": ("tiny_qwen3", ("random", 14, [4, 6]), 12, True, True),
    "tiny_bias_seq": ("tiny_bias", ("random", 15, [5, 3]), 10, False, False),
    "mid_seq": ("mid", ("random", 16, [20, 37, 64]), 24, False, False),
    "mid_tree": ("mid", ("random", 16, [20, 37, 64]), 24, True, False),
    # Constructed coverage vector: exact lm_head tie (rows 5 and 17) and a
    # subnormal step-0 logit (row 29); the prompt is synth.coverage_prompt().
    "coverage_seq": ("coverage", ("random", 20261016, [4]), 12, False, False),
    "coverage_tree": ("coverage", ("random", 20261016, [4]), 12, True, False),
    # BASELINE configurations (full sizes; C5 on a seeded subset).
    "c1": ("smollm2", ("workload", "c1", 0, 1), 256, False, False),
    "c1_tree": ("smollm2", ("workload", "c1", 0, 1), 256, True, False),
    "c2": ("smollm2", ("workload", "c2", 0, 64), 256, False, False),
    "c2_tree": ("smollm2", ("workload", "c2", 0, 64), 256, True, False),
    "c3": ("llama160m", ("workload", "c3", 0, 300), 128, False, False),
    "c3_tree": ("llama160m", ("workload", "c3", 0, 300), 128, True, False),
    "c4": ("qwen3_0p6b", ("workload", "c4", 0, 32), 256, False, True),
    "c4_tree": ("qwen3_0p6b", ("workload", "c4", 0, 32), 256, True, True),
    "c5_subset": ("smollm2", ("workload", "c5", 0, 4), 1024, False, False),
    # The sequences other ranks decode in the multi-GPU runs: C2 weak scaling
    # gives rank r sequences 64r .. 64r+63 (r < 8); C5 strong scaling over 8
    # GPUs gives rank r sequences 32r .. 32r+31, checked here at 32r + 5.
    "c2_shards": ("smollm2", ("workload", "c2", 64, 448), 256, False, False),
    # Tree mode on the other two head shapes of the decode kernels (head size
    # 64 with one query head per KV head; head size 128, two per KV head, with
    # the Qwen3 q/k norm): the first sequences of C3 and C4, 16 tokens.
    "tree_llama160m": ("llama160m", ("workload", "c3", 0, 4), 16, True, False),
    "tree_qwen3": ("qwen3_0p6b", ("workload", "c4", 0, 2), 16, True, True),
    "c5_spread": ("smollm2", ("workload_idx", "c5", [37, 69, 101, 133, 165, 197, 229]), 1024, False, False),
}


def build_prompts(model: str, spec) -> list:
    if spec[0] == "workload":
        _, w, first, count = spec
        return list(synth.prompt_ids(w, n_seq=count, first=first))
    if spec[0] == "workload_idx":
        _, w, idx = spec
        return [synth.prompt_ids(w, n_seq=1, first=i)[0] for i in idx]
    _, seed, lens = spec
    return [synth.random_prompts(model, 1, L, seed, first=i)[0] for i, L in enumerate(lens)]


def run_case(name: str, root: str, workers: int) -> dict:
    model, spec, gen, tree, sampled = CASES[name]
    d = synth.ensure_model(model, root)
    prompts = build_prompts(model, spec)
    t0 = time.time()
    res = pyoracle.run_refdrv(d, prompts, gen, tree=tree, sample=SAMPLE if sampled else None,
                              step_digests=True, workers=workers)
    seqs = []
    for i, r in enumerate(res):
        e = {"witness": r["witness"], "argmax": r["argmax"], "steps_sha": r["steps_sha"],
             "tokens_sha": hashlib.sha256(b"".join(int(t).to_bytes(4, "little") for t in r["tokens"])).hexdigest()}
        if i == 0:
            e["tokens"] = r["tokens"]
            e["step_digests"] = r["step_digests"]
        seqs.append(e)
    with open(os.path.join(d, "config.json"), "rb") as f:
        cfg_sha = hashlib.sha256(f.read()).hexdigest()
    out = {"case": name, "model": model, "prompts": list(spec), "gen": gen,
           "reduction": "tree" if tree else "sequential", "sample": SAMPLE if sampled else None,
           "config_sha256": cfg_sha, "weights_sha256": pyoracle.artifact_hashes(d)[:32].hex(),
           "generator": "oracle/_ref/" + os.path.basename(pyoracle.refdrv_path(qwen3="head_dim" in
                                                                                pyoracle.read_config(d),
                                                                                tree=tree)),
           "cpu_seconds": round(time.time() - t0, 1), "sequences": seqs}
    with open(os.path.join(HERE, name + ".json"), "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("cases", nargs="*", default=None)
    ap.add_argument("--workers", type=int, default=os.cpu_count() or 1)
    ap.add_argument("--root", default=synth.default_root())
    a = ap.parse_args()
    names = a.cases or list(CASES)
    for n in names:
        t = time.time()
        run_case(n, a.root, a.workers)
        print(f"{n}: {time.time() - t:.1f}s", flush=True)


if __name__ == "__main__":
    main()
