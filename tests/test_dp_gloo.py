"""Data-parallel host logic on CPU: two gloo ranks.

Each rank computes oracle gradients on its own micro-batch, permutes them to
the trainer's layer-major layout, all-reduces them bucket by bucket in the
order llmk_gpt2_dp_buckets gives, and scales by 1/world as llmk_gpt2_update
does. The result must equal the gradient of the mean loss over the
concatenated batch computed in one process. A second case makes one rank
fail before its collective and checks that the other rank's collective ends
with an error inside the process-group timeout instead of hanging.
"""
import ctypes as C
import datetime
import os
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SMALL = dict(max_seq_len=32, vocab_size=97, padded_vocab_size=128, num_layers=2, num_heads=2, channels=128)
B, T = 2, 16


def _setup_paths():
    for p in (ROOT, os.path.join(ROOT, "llm.cpp_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _rank_grads(rank, params, toks):
    import oracle as O
    cfg = O.config(**SMALL)
    m = O.Model(cfg, params, B, T)
    chunk = toks[rank * B * T:(rank + 1) * B * T + 1]
    m.forward(chunk[:-1], chunk[1:])
    m.zero_grad()
    m.backward()
    return m.grads()


def _worker(rank, world, port, params, toks, out_q):
    _setup_paths()
    import torch
    import torch.distributed as dist
    import llmk
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    g = _rank_grads(rank, params, toks)
    cfg = llmk.GPT2Config(**SMALL)
    lm = np.empty_like(g)
    llmk.call("llmk_gpt2_to_layer_major", C.byref(cfg), g.ctypes.data, lm.ctypes.data, 0)
    n = llmk.lib().llmk_gpt2_dp_buckets(C.byref(cfg), None, 0)
    arr = (C.c_size_t * (2 * n))()
    llmk.lib().llmk_gpt2_dp_buckets(C.byref(cfg), arr, n)
    t = torch.from_numpy(lm)
    for i in range(n):
        b, e = arr[2 * i], arr[2 * i + 1]
        dist.all_reduce(t[b:e], op=dist.ReduceOp.SUM)
    t /= world
    back = np.empty_like(lm)
    llmk.call("llmk_gpt2_to_layer_major", C.byref(cfg), t.numpy().ctypes.data, back.ctypes.data, 1)
    out_q.put((rank, back))
    dist.barrier()
    dist.destroy_process_group()


def _failing_worker(rank, world, port, out_q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        # this rank fails between steps: it never joins the collective
        out_q.put((rank, "exited"))
        out_q.close()
        out_q.join_thread()  # flush the queue before the hard exit
        os._exit(0)
    try:
        dist.all_reduce(torch.ones(1024))
        out_q.put((rank, "completed"))
    except Exception as e:  # the surviving rank must see an error, not hang
        out_q.put((rank, f"error: {type(e).__name__}"))


def _free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_bucketed_allreduce_matches_full_batch():
    _setup_paths()
    import oracle as O
    cfg = O.config(**SMALL)
    params = O.init_params(cfg, 3)
    world = 2
    toks = O.tokens(world * B * T + 1, cfg.vocab_size, 3)
    # reference: one process, both micro-batches, mean of the two gradients
    ref = (_rank_grads(0, params, toks) + _rank_grads(1, params, toks)) / 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, params, toks, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        np.testing.assert_allclose(res[r], ref, rtol=1e-5, atol=1e-7)


def test_rank_failure_surfaces_as_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=90) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "exited"
    assert res[0].startswith("error"), res[0]
