"""Data-parallel training on 2 GPUs: NCCL gradient all-reduce inside the trainer.

Two ranks (one process per GPU, torch.distributed only to share the NCCL id)
each run one step of a small GPT-2 on their own micro-batch. After
llmk_gpt2_backward the gradient buffer holds the SUM over ranks (AdamW applies
the 1/world average), so it must equal the oracle's gradients of micro-batch
0 plus micro-batch 1, and both ranks must hold identical parameters after the
update. Needs 2 GPUs; skipped otherwise. NVLS is disabled (NCCL_NVLS_ENABLE=0).
"""
import datetime
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SMALL = dict(max_seq_len=128, vocab_size=1000, padded_vocab_size=1024, num_layers=2, num_heads=2, channels=128)
B, T = 2, 128


def _paths():
    for p in (ROOT, os.path.join(ROOT, "llm.cpp_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _worker(rank, world, port, params, toks, q):
    _paths()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    import llmk
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    m = llmk.GPT2(B, T, math=llmk.MATH_TF32, **SMALL)
    m.load_parameters(params)
    obj = [llmk.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    m.enable_dp(obj[0], rank, world)
    chunk = toks[rank * B * T:(rank + 1) * B * T + 1]
    m.train_step(chunk[:-1], chunk[1:], 3e-4, t=1)
    m.synchronize(timeout_ms=60000)
    q.put((rank, m.read_gradients(), m.read_parameters()))
    dist.barrier()
    m.close()
    dist.destroy_process_group()


def test_two_gpu_gradient_allreduce():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _paths()
    import oracle as O
    cfg = O.config(**SMALL)
    params = O.init_params(cfg, 21)
    toks = O.tokens(2 * B * T + 1, cfg.vocab_size, 21)
    ref = np.zeros(sum(O.param_sizes(cfg)), np.float64)
    for r in range(2):
        mo = O.Model(cfg, params, B, T)
        c = toks[r * B * T:(r + 1) * B * T + 1]
        mo.forward(c[:-1], c[1:])
        mo.zero_grad()
        mo.backward()
        ref += mo.grads()
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, params, toks, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, g, p = q.get(timeout=300)
        res[r] = (g, p)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(2):
        g = res[r][0].astype(np.float64)
        err = np.linalg.norm(g - ref) / np.linalg.norm(ref)
        assert err < 1e-2, (r, err)
    assert np.array_equal(res[0][1], res[1][1]), "ranks diverged after the update"
