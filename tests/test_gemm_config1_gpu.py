"""Configuration 1 of the benchmark spec at its full size: the GPT-2 124M
layer GEMMs at BT = 8192 rows (QKV 768->2304, attention projection 768->768,
FC 768->3072, FC projection 3072->768, tied lm_head 768->50304), forward
(with bias, except the lm_head), input gradient, weight gradient (K = BT)
and bias gradient, in TF32 and BF16 modes, through llmk_matmul_forward /
llmk_matmul_backward — checked against the oracle's matmul (the reference's
MatMulForward / MatMulBackward, gpt2/matmul.cpp:15-71).

At this size a full fp32 CPU product of the lm_head alone is ~1.9 TFLOP, so
the oracle evaluates SAMPLED outputs exactly: 64 seeded rows of the forward
output and of the input gradient (the oracle run on those rows of the input
and output gradient), and 64 seeded output features of the weight and bias
gradients (the oracle's backward over all 8192 rows for those features).
The device computes the full outputs; the planner's choices at this size
(split-K factors, 256-wide CTA-pair tiles, the lm_head raster) are the ones
under test. Inputs are N(0, 1) from the oracle's seeded generator; the
device gets them rounded to bf16 in BF16 mode, the oracle the fp32 values
(the reference's fp32 path on the same seeded inputs). Bars: max relative
error 1e-2 (BF16), 2e-3 (TF32).
"""
import numpy as np
import pytest

import oracle as O
from conftest import max_rel_err

pytestmark = pytest.mark.gpu

BT = 8192
SHAPES = [("qkv", 768, 2304), ("attproj", 768, 768), ("fc", 768, 3072), ("fcproj", 3072, 768),
          ("lm_head", 768, 50304)]


@pytest.mark.parametrize("mathname,tol", [("bf16", 1e-2), ("tf32", 2e-3)])
@pytest.mark.parametrize("name,IC,OC", SHAPES)
def test_config1_gemm_forms_vs_oracle(cuda_dev, mathname, tol, name, IC, OC):
    import torch
    import llmk
    math = llmk.MATH_BF16 if mathname == "bf16" else llmk.MATH_TF32
    dt = torch.bfloat16 if mathname == "bf16" else torch.float32
    seed = 100 + 10 * [s[0] for s in SHAPES].index(name)
    has_bias = name != "lm_head"
    x = O.normal((BT, IC), seed + 1)
    W = O.normal((OC, IC), seed + 2)
    b = O.normal((OC,), seed + 3)
    dout = O.normal((BT, OC), seed + 4)
    s = llmk.stream_ptr()
    xd = torch.from_numpy(x).to(cuda_dev).to(dt)
    Wd = torch.from_numpy(W).to(cuda_dev).to(dt)
    dd = torch.from_numpy(dout).to(cuda_dev).to(dt)
    bd = torch.from_numpy(b).to(cuda_dev) if has_bias else None
    out = torch.empty(BT, OC, device=cuda_dev)
    llmk.call("llmk_matmul_forward", out.data_ptr(), llmk.F32, xd.data_ptr(), Wd.data_ptr(), llmk.ptr(bd), BT, IC,
              OC, math, s)
    dinp = torch.empty(BT, IC, device=cuda_dev)
    dW = torch.empty(OC, IC, device=cuda_dev)
    db = torch.empty(OC, device=cuda_dev)
    wsb = llmk.lib().llmk_matmul_backward_workspace(BT, IC, OC, math)
    ws = torch.empty(wsb // 4 + 64, device=cuda_dev)
    # overwrite semantics (flags 0): every element is produced by this call
    llmk.call("llmk_matmul_backward", dinp.data_ptr(), llmk.F32, dW.data_ptr(), db.data_ptr() if has_bias else None,
              dd.data_ptr(), xd.data_ptr(), Wd.data_ptr(), BT, IC, OC, math, 0, ws.data_ptr(), wsb, s)
    rng = np.random.default_rng(seed)
    rows = np.sort(rng.choice(BT, 64, replace=False))
    feats = np.sort(rng.choice(OC, 64, replace=False))
    # forward rows
    y_ref = np.zeros((64, OC), np.float32)
    xr = np.ascontiguousarray(x[rows])
    O.orc().orc_matmul_forward(y_ref, xr, W, b.ctypes.data if has_bias else None, 64, IC, OC)
    # input-gradient rows (the oracle accumulates into zeros)
    di_ref = np.zeros((64, IC), np.float32)
    dW_scratch = np.zeros((OC, IC), np.float32)
    O.orc().orc_matmul_backward(di_ref, dW_scratch, None, np.ascontiguousarray(dout[rows]), xr, W, 64, IC, OC)
    # weight- and bias-gradient features over all BT rows
    dW_ref = np.zeros((64, IC), np.float32)
    db_ref = np.zeros(64, np.float32)
    di_scratch = np.zeros((BT, IC), np.float32)
    O.orc().orc_matmul_backward(di_scratch, dW_ref, db_ref.ctypes.data, np.ascontiguousarray(dout[:, feats]), x,
                                np.ascontiguousarray(W[feats]), BT, IC, 64)
    torch.cuda.synchronize()
    rows_t = torch.from_numpy(rows).to(cuda_dev)
    feats_t = torch.from_numpy(feats).to(cuda_dev)
    errs = {"fwd": max_rel_err(out.index_select(0, rows_t).cpu(), y_ref),
            "dinp": max_rel_err(dinp.index_select(0, rows_t).cpu(), di_ref),
            "dweight": max_rel_err(dW.index_select(0, feats_t).cpu(), dW_ref)}
    if has_bias:
        errs["dbias"] = max_rel_err(db.index_select(0, feats_t).cpu(), db_ref)
    print(mathname, name, {k: f"{v:.2e}" for k, v in errs.items()})
    for k, v in errs.items():
        assert v < tol, (k, v)
    assert llmk.device_status() == 0
