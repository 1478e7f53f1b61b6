"""Multi-process host logic on CPU (gloo, world size 2): the sequence
sharding bench.py uses and the one exchange step (bench.gather_outputs:
tokens, per-step digests, witness and argmax digests) reproduce a
single-process run exactly."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def test_shard_covers_every_sequence_once():
    for n in (1, 7, 64, 300):
        for w in (1, 2, 3, 4, 8):
            seen = []
            for r in range(w):
                f, c = bench.shard(n, w, r)
                seen += list(range(f, f + c))
            assert seen == list(range(n))
    # C3: 300 sequences over 8 GPUs -> 38,38,38,38,37,37,37,37
    assert [bench.shard(300, 8, r)[1] for r in range(8)] == [38] * 4 + [37] * 4


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_q):
    import importlib
    import torch
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    import sys
    sys.path.insert(0, os.path.join(root, "oracle"))
    import pyoracle
    synth = importlib.import_module("cis2-lab-archive_b200.synth")
    d = synth.ensure_model("tiny", synth.default_root())
    n_total = 5
    first, cnt = bench.shard(n_total, world, rank)
    prompts = [synth.random_prompts("tiny", 1, 4 + i, 31, first=i)[0] for i in range(first, first + cnt)]
    r = pyoracle.PortOracle(d).generate(prompts, 6)
    counts = [bench.shard(n_total, world, q)[1] for q in range(world)]
    got = bench.gather_outputs(r, 6, counts, "cpu")
    if rank == 0:
        out_q.put({k: np.array(v) for k, v in got.items()})
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_sharded_gather_equals_single_run(synth, synth_root, oracle):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    d = synth.ensure_model("tiny", synth_root)
    prompts = [synth.random_prompts("tiny", 1, 4 + i, 31, first=i)[0] for i in range(5)]
    want = oracle.PortOracle(d).generate(prompts, 6)
    for k in ("tokens", "step_digests", "witness", "argmax"):
        assert np.array_equal(got[k], want[k]), k


def test_failed_rank_is_detected_on_host(tmp_path):
    """A rank that never joins: the other rank's rendezvous ends with an
    error after its timeout instead of hanging (failure is made on the host)."""
    import datetime
    port = _free_port()
    store = dist.TCPStore("127.0.0.1", port, world_size=2, is_master=True,
                          timeout=datetime.timedelta(seconds=2), wait_for_workers=False)
    with pytest.raises(Exception):
        dist.init_process_group("gloo", store=store, rank=0, world_size=2,
                                timeout=datetime.timedelta(seconds=2))
    if dist.is_initialized():
        dist.destroy_process_group()
