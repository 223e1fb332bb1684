"""Fused lm_head + softmax / cross-entropy (llmk_matmul_crossentropy_forward,
llmk_matmul_softmax_forward) vs the oracle, and vs the unfused GPU path
(llmk_gemm + llmk_softmax_crossentropy) on the same operands.

Oracle: the reference CPU algorithm (matmul forward, softmax over the first V
columns, cross-entropy, CrossEntropySoftmaxBackward) on the operands as the
device sees them (bf16-rounded in bf16 mode). Tolerances: bf16 1e-2, TF32
2e-3 max-relative; fused vs unfused on the device (same logits bits, other
reduction order): losses 1e-5, dlogits one bf16 step of the largest value."""
import numpy as np
import pytest

import oracle as O
from conftest import max_rel_err

pytestmark = pytest.mark.gpu

SHAPES = [(333, 128, 1001, 1008), (1024, 256, 4000, 4096), (256, 768, 50257, 50304)]


def _operands(BT, C, V, Vp, seed, mathname, bias=False):
    import torch
    x = O.normal((BT, C), seed, std=1.0)
    W = O.normal((Vp, C), seed + 1, std=0.1)  # logits of std 1-3, as a trained lm_head gives
    W[V:] = 0.0  # padded vocabulary rows are zero, as in the model
    b = O.normal((Vp,), seed + 2) if bias else None
    tgt = O.tokens(BT, V, seed + 3)
    if mathname == "bf16":
        x = torch.from_numpy(x).bfloat16().float().numpy()
        W = torch.from_numpy(W).bfloat16().float().numpy()
    return x, W, b, tgt


def _oracle(x, W, b, tgt, BT, C, V, Vp, dtname):
    import torch
    logits = np.zeros((BT, Vp), np.float32)
    O.orc().orc_matmul_forward(logits, x, W, None if b is None else b.ctypes.data, BT, C, Vp)
    if dtname == "bf16":  # the device stores bf16 logits and normalises those
        logits = torch.from_numpy(logits).bfloat16().float().numpy()
    probs = np.zeros((BT, V), np.float32)
    O.orc().orc_softmax(probs, logits, BT, V, Vp)
    lo = np.zeros(BT, np.float32)
    O.orc().orc_cross_entropy(lo.ctypes.data, probs, tgt, BT, V)
    dlo = np.zeros((BT, Vp), np.float32)
    O.orc().orc_cross_entropy_softmax_backward(dlo, probs, tgt, BT, V, Vp)
    return logits, probs, lo, dlo


@pytest.mark.parametrize("mathname,tol", [("bf16", 1e-2), ("tf32", 2e-3)])
@pytest.mark.parametrize("shape", SHAPES)
def test_matmul_crossentropy_vs_oracle_and_unfused(cuda_dev, mathname, tol, shape):
    import torch
    import llmk
    BT, C, V, Vp = shape
    math = llmk.MATH_BF16 if mathname == "bf16" else llmk.MATH_TF32
    dt = torch.bfloat16 if mathname == "bf16" else torch.float32
    x, W, _, tgt = _operands(BT, C, V, Vp, 61, mathname)
    xd, Wd = torch.from_numpy(x).to(cuda_dev, dt), torch.from_numpy(W).to(cuda_dev, dt)
    tg = torch.from_numpy(tgt).to(cuda_dev)
    s = llmk.stream_ptr()
    ws = torch.empty(llmk.lib().llmk_matmul_softmax_workspace(BT, Vp), dtype=torch.uint8, device=cuda_dev)
    # fused: logits overwritten by dlogits
    fused = torch.empty(BT, Vp, dtype=dt, device=cuda_dev)
    losses = torch.empty(BT, device=cuda_dev)
    llmk.call("llmk_matmul_crossentropy_forward", losses.data_ptr(), fused.data_ptr(), llmk.dtype_code(fused),
              xd.data_ptr(), Wd.data_ptr(), None, tg.data_ptr(), BT, C, Vp, V, 1.0 / BT, 1, math, ws.data_ptr(),
              ws.numel(), s)
    # losses only: the logits stay
    keep = torch.empty(BT, Vp, dtype=dt, device=cuda_dev)
    losses_k = torch.empty(BT, device=cuda_dev)
    llmk.call("llmk_matmul_crossentropy_forward", losses_k.data_ptr(), keep.data_ptr(), llmk.dtype_code(keep),
              xd.data_ptr(), Wd.data_ptr(), None, tg.data_ptr(), BT, C, Vp, V, 1.0 / BT, 0, math, ws.data_ptr(),
              ws.numel(), s)
    # unfused on the device: GEMM, then the two-pass softmax + cross-entropy
    unf = torch.empty(BT, Vp, dtype=dt, device=cuda_dev)
    llmk.gemm(unf, xd, Wd, math=math)
    logits_dev = unf.clone()
    losses_u = torch.empty(BT, device=cuda_dev)
    llmk.call("llmk_softmax_crossentropy", losses_u.data_ptr(), unf.data_ptr(), unf.data_ptr(), llmk.dtype_code(unf),
              tg.data_ptr(), BT, V, Vp, 1.0 / BT, s)
    torch.cuda.synchronize()
    assert llmk.device_status() == 0
    _, _, lo, dlo = _oracle(x, W, None, tgt, BT, C, V, Vp, mathname)
    assert max_rel_err(losses.cpu(), lo) < tol
    assert max_rel_err(fused.float().cpu(), dlo) < tol
    assert torch.count_nonzero(fused[:, V:]).item() == 0
    # same logits as the plain GEMM, bit for bit; losses as the unfused pass
    assert torch.equal(keep, logits_dev)
    assert torch.equal(losses_k, losses)
    assert max_rel_err(losses.cpu(), losses_u.cpu()) < 1e-5
    step = 2.0 ** -7 if mathname == "bf16" else 1e-5
    assert max_rel_err(fused.float().cpu(), unf.float().cpu()) <= step


@pytest.mark.parametrize("mathname,tol", [("bf16", 1e-2), ("tf32", 2e-3)])
@pytest.mark.parametrize("alias", [False, True])
def test_matmul_softmax_forward(cuda_dev, mathname, tol, alias):
    """gpt2cuda::BatchMatmulNTSoftmaxForward counterpart, with a bias: the
    logits and the probabilities (0 on the padded columns), probabilities
    written over the logits when aliased."""
    import torch
    import llmk
    BT, C, V, Vp = 600, 192, 3001, 3008
    math = llmk.MATH_BF16 if mathname == "bf16" else llmk.MATH_TF32
    dt = torch.bfloat16 if mathname == "bf16" else torch.float32
    x, W, b, _ = _operands(BT, C, V, Vp, 71, mathname, bias=True)
    xd, Wd = torch.from_numpy(x).to(cuda_dev, dt), torch.from_numpy(W).to(cuda_dev, dt)
    bd = torch.from_numpy(b).to(cuda_dev)
    ws = torch.empty(llmk.lib().llmk_matmul_softmax_workspace(BT, Vp), dtype=torch.uint8, device=cuda_dev)
    logits = torch.empty(BT, Vp, dtype=dt, device=cuda_dev)
    probs = logits if alias else torch.empty(BT, Vp, dtype=dt, device=cuda_dev)
    llmk.call("llmk_matmul_softmax_forward", probs.data_ptr(), logits.data_ptr(), llmk.dtype_code(logits),
              xd.data_ptr(), Wd.data_ptr(), bd.data_ptr(), BT, C, Vp, V, math, ws.data_ptr(), ws.numel(),
              llmk.stream_ptr())
    torch.cuda.synchronize()
    assert llmk.device_status() == 0
    lref, pref, _, _ = _oracle(x, W, b, np.zeros(BT, np.int32), BT, C, V, Vp, mathname)
    if not alias:
        assert max_rel_err(logits.float().cpu(), lref) < tol
    assert max_rel_err(probs[:, :V].float().cpu(), pref) < tol
    assert torch.count_nonzero(probs[:, V:]).item() == 0
    rows = probs[:, :V].float().sum(dim=1)
    assert torch.allclose(rows, torch.ones_like(rows), atol=2e-2 if mathname == "bf16" else 1e-4)


def test_matmul_crossentropy_bad_target_and_arguments(cuda_dev):
    """A target outside [0, V) gives a NaN loss for that row only; a missing
    or short workspace is refused before any launch."""
    import torch
    import llmk
    BT, C, V, Vp = 64, 64, 500, 512
    x, W, _, tgt = _operands(BT, C, V, Vp, 81, "bf16")
    tgt[5] = V + 3
    tgt[9] = -1
    xd, Wd = torch.from_numpy(x).to(cuda_dev, torch.bfloat16), torch.from_numpy(W).to(cuda_dev, torch.bfloat16)
    tg = torch.from_numpy(tgt).to(cuda_dev)
    n = llmk.lib().llmk_matmul_softmax_workspace(BT, Vp)
    ws = torch.empty(n, dtype=torch.uint8, device=cuda_dev)
    lg = torch.empty(BT, Vp, dtype=torch.bfloat16, device=cuda_dev)
    losses = torch.empty(BT, device=cuda_dev)
    args = (losses.data_ptr(), lg.data_ptr(), llmk.BF16, xd.data_ptr(), Wd.data_ptr(), None, tg.data_ptr(), BT, C, Vp,
            V, 1.0 / BT, 1, llmk.MATH_BF16)
    with pytest.raises(llmk.LlmkError) as e:
        llmk.call("llmk_matmul_crossentropy_forward", *args, ws.data_ptr(), n - 8, llmk.stream_ptr())
    assert e.value.code == 5
    llmk.call("llmk_matmul_crossentropy_forward", *args, ws.data_ptr(), n, llmk.stream_ptr())
    torch.cuda.synchronize()
    bad = torch.isnan(losses.cpu())
    assert bad[5] and bad[9] and int(bad.sum()) == 2
    assert llmk.device_status() == 0
