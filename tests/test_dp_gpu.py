"""Data-parallel training on 2 GPUs: NCCL gradient all-reduce inside the trainer.

Two ranks (one process per GPU, torch.distributed only to share the NCCL id
and the per-step losses) each train on their own micro-batch.

test_two_gpu_gradient_allreduce (TF32, eager, one step): after
llmk_gpt2_backward the gradient buffer holds the SUM over ranks (AdamW applies
the 1/world average), so it must equal the oracle's gradients of micro-batch
0 plus micro-batch 1, and both ranks must hold identical parameters after the
update.

test_two_gpu_matches_one_gpu_concatenated (bf16 and TF32, CUDA-graph replay,
3 steps — the benchmark's mode): the mean of the ranks' losses at every step
equals the loss of ONE GPU training on the concatenated batch (B = 2 * B per
rank) within 1e-3 relative, the ranks' parameters are bit-identical after
every step, and the parameters match the one-GPU run's (mean absolute
difference below 1e-5).

Needs 2 GPUs; skipped otherwise. NVLS is disabled (NCCL_NVLS_ENABLE=0).
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
STEPS = 3


def _paths():
    for p in (ROOT, os.path.join(ROOT, "llm.cpp_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _worker(rank, world, port, params, toks, q, math, graph, steps):
    _paths()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    import llmk
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    m = llmk.GPT2(B, T, math=math, **SMALL)
    m.load_parameters(params)
    obj = [llmk.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    m.enable_dp(obj[0], rank, world)
    m.use_graph(graph)
    losses, snaps = [], []
    for s in range(steps):
        chunk = toks[s][rank * B * T:(rank + 1) * B * T + 1]
        losses.append(m.train_step(chunk[:-1], chunk[1:], 1e-3, t=s + 1))
        m.synchronize(timeout_ms=60000)
        snaps.append(m.read_parameters())
    q.put((rank, m.read_gradients(), losses, snaps))
    dist.barrier()
    m.close()
    dist.destroy_process_group()


def _run_two(params, toks, math, graph, steps):
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, params, toks, q, math, graph, steps)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, g, losses, snaps = q.get(timeout=300)
        res[r] = (g, losses, snaps)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


def test_two_gpu_gradient_allreduce():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _paths()
    import llmk
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
    res = _run_two(params, [toks], llmk.MATH_TF32, False, 1)
    for r in range(2):
        g = res[r][0].astype(np.float64)
        err = np.linalg.norm(g - ref) / np.linalg.norm(ref)
        assert err < 1e-2, (r, err)
    assert np.array_equal(res[0][2][-1], res[1][2][-1]), "ranks diverged after the update"


@pytest.mark.parametrize("mathname", ["bf16", "tf32"])
def test_two_gpu_matches_one_gpu_concatenated(mathname):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _paths()
    import llmk
    import oracle as O
    math = llmk.MATH_BF16 if mathname == "bf16" else llmk.MATH_TF32
    cfg = O.config(**SMALL)
    params = O.init_params(cfg, 23)
    toks = [O.tokens(2 * B * T + 1, cfg.vocab_size, 23 + s) for s in range(STEPS)]
    res = _run_two(params, toks, math, True, STEPS)
    # one GPU, the two micro-batches side by side (2B sequences), same steps
    torch.cuda.set_device(0)
    m = llmk.GPT2(2 * B, T, math=math, **SMALL)
    m.load_parameters(params)
    m.use_graph(True)
    single, single_p = [], []
    for s in range(STEPS):
        c = toks[s]
        # rank r's sequences are tokens [r*B*T, (r+1)*B*T] (targets shifted by one within each chunk)
        inp = np.concatenate([c[r * B * T:(r + 1) * B * T] for r in range(2)])
        tgt = np.concatenate([c[r * B * T + 1:(r + 1) * B * T + 1] for r in range(2)])
        single.append(m.train_step(inp, tgt, 1e-3, t=s + 1))
        single_p.append(m.read_parameters())
    m.close()
    for s in range(STEPS):
        mean = 0.5 * (res[0][1][s] + res[1][1][s])
        assert abs(mean - single[s]) / single[s] < 1e-3, (s, mean, single[s])
        assert np.array_equal(res[0][2][s], res[1][2][s]), f"ranks diverged at step {s}"
        # AdamW moves each parameter by at most lr per step, whatever the
        # gradient's size, so a sign flip of a near-zero gradient (reduction
        # order) can differ by 2 * lr per step; on average they agree closely
        d = np.abs(res[0][2][s].astype(np.float64) - single_p[s].astype(np.float64))
        assert d.max() <= 2e-3 * (s + 1) + 1e-6, (s, d.max())
        assert d.mean() < 1e-5, (s, d.mean())
