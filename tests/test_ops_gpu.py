"""Linear-layer and bandwidth-bound entry points vs the oracle (reference CPU algorithm).

Every case feeds the device and the oracle the same seeded bytes. BF16
results: max relative error 1e-2; TF32: 2e-3; fp32 bandwidth kernels: 1e-5
(1e-4 where a reduction order differs).
"""
import numpy as np
import pytest

import oracle as O
from conftest import max_rel_err

pytestmark = pytest.mark.gpu


def T(x, dev, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return t.to(dtype) if dtype is not None else t


def bf(x):
    import torch
    return torch.from_numpy(x).bfloat16().float().numpy()


@pytest.mark.parametrize("mathname,tol", [("bf16", 1e-2), ("tf32", 2e-3)])
@pytest.mark.parametrize("BT,C,OC", [(512, 768, 2304), (256, 3072, 768), (384, 768, 50304)])
def test_matmul_forward_backward_vs_oracle(cuda_dev, mathname, tol, BT, C, OC):
    import torch
    import llmk
    math = llmk.MATH_BF16 if mathname == "bf16" else llmk.MATH_TF32
    dt = torch.bfloat16 if mathname == "bf16" else torch.float32
    x = O.normal((BT, C), 1)
    W = O.normal((OC, C), 2)
    b = O.normal((OC,), 3)
    dout = O.normal((BT, OC), 4)
    has_bias = OC != 50304  # the tied lm_head has no bias
    s = llmk.stream_ptr()
    xd, Wd, dd = T(x, cuda_dev, dt), T(W, cuda_dev, dt), T(dout, cuda_dev, dt)
    bd = T(b, cuda_dev) if has_bias else None
    out = T(np.zeros((BT, OC), np.float32), cuda_dev)
    llmk.call("llmk_matmul_forward", out.data_ptr(), llmk.F32, xd.data_ptr(), Wd.data_ptr(), llmk.ptr(bd), BT, C, OC,
              math, s)
    y = np.zeros((BT, OC), np.float32)
    O.orc().orc_matmul_forward(y, x, W, b.ctypes.data if has_bias else None, BT, C, OC)
    torch.cuda.synchronize()
    assert max_rel_err(out.cpu(), torch.from_numpy(y)) < tol
    # backward with the reference's accumulate semantics on dinp / dweight
    dinp0 = O.normal((BT, C), 5)
    dW0 = O.normal((OC, C), 6)
    dinp = T(dinp0, cuda_dev)
    dW = T(dW0, cuda_dev)
    db = T(np.zeros(OC, np.float32), cuda_dev)
    ws_b = llmk.lib().llmk_matmul_backward_workspace(BT, C, OC, math)
    ws = torch.empty(ws_b // 4 + 64, device=cuda_dev)
    flags = llmk.ACCUM_DINP | llmk.ACCUM_DWEIGHT
    llmk.call("llmk_matmul_backward", dinp.data_ptr(), llmk.F32, dW.data_ptr(), db.data_ptr() if has_bias else None,
              dd.data_ptr(), xd.data_ptr(), Wd.data_ptr(), BT, C, OC, math, flags, ws.data_ptr(), ws_b, s)
    di_o, dW_o, db_o = dinp0.copy(), dW0.copy(), np.zeros(OC, np.float32)
    O.orc().orc_matmul_backward(di_o, dW_o, db_o.ctypes.data, dout, x, W, BT, C, OC)
    torch.cuda.synchronize()
    assert max_rel_err(dinp.cpu(), torch.from_numpy(di_o)) < tol
    assert max_rel_err(dW.cpu(), torch.from_numpy(dW_o)) < tol
    if has_bias:
        ref_db = db_o if mathname == "tf32" else bf(dout).sum(0)
        assert max_rel_err(db.cpu(), torch.from_numpy(ref_db)) < (1e-5 if mathname == "bf16" else tol)
    assert llmk.device_status() == 0


def test_layernorm_vs_oracle(cuda_dev):
    import torch
    import llmk
    N, C = 1000, 768
    x = O.normal((N, C), 11, std=2.0)
    g = O.normal((C,), 12)
    be = O.normal((C,), 13)
    dy = O.normal((N, C), 14)
    s = llmk.stream_ptr()
    xd, gd, bd = T(x, cuda_dev), T(g, cuda_dev), T(be, cuda_dev)
    y = torch.empty(N, C, device=cuda_dev)
    yb = torch.empty(N, C, device=cuda_dev, dtype=torch.bfloat16)
    mean = torch.empty(N, device=cuda_dev)
    rstd = torch.empty(N, device=cuda_dev)
    llmk.call("llmk_layernorm_forward", y.data_ptr(), llmk.F32, mean.data_ptr(), rstd.data_ptr(), xd.data_ptr(),
              gd.data_ptr(), bd.data_ptr(), N, C, s)
    llmk.call("llmk_layernorm_forward", yb.data_ptr(), llmk.BF16, None, None, xd.data_ptr(), gd.data_ptr(),
              bd.data_ptr(), N, C, s)
    yo = np.zeros_like(x)
    mo = np.zeros(N, np.float32)
    ro = np.zeros(N, np.float32)
    O.orc().orc_layernorm_forward(yo, mo.ctypes.data, ro.ctypes.data, x, g, be, N, C)
    torch.cuda.synchronize()
    assert max_rel_err(y.cpu(), torch.from_numpy(yo)) < 1e-5
    assert max_rel_err(yb.float().cpu(), torch.from_numpy(yo)) < 1e-2
    assert max_rel_err(rstd.cpu(), torch.from_numpy(ro)) < 1e-5
    # backward: dinp accumulate, dgamma/dbeta accumulate, bf16 copy
    d0 = O.normal((N, C), 15)
    dinp = T(d0, cuda_dev)
    dinp_b = torch.empty(N, C, device=cuda_dev, dtype=torch.bfloat16)
    dg = T(np.ones(C, np.float32), cuda_dev)
    db = T(np.ones(C, np.float32), cuda_dev)
    ws_b = llmk.lib().llmk_layernorm_backward_workspace(N, C)
    ws = torch.empty(ws_b // 4 + 64, device=cuda_dev)
    dyd = T(dy, cuda_dev)
    dsum = torch.full((C,), float("nan"), device=cuda_dev)
    llmk.call("llmk_layernorm_backward", dinp.data_ptr(), dinp_b.data_ptr(), dg.data_ptr(), db.data_ptr(),
              dsum.data_ptr(), dyd.data_ptr(), llmk.F32, xd.data_ptr(), gd.data_ptr(), mean.data_ptr(),
              rstd.data_ptr(), N, C, llmk.ACCUM_DINP | llmk.ACCUM_DPARAM, ws.data_ptr(), ws_b, s)
    dxo = np.zeros_like(x)
    dgo = np.ones(C, np.float32)
    dbo = np.ones(C, np.float32)
    O.orc().orc_layernorm_backward(dxo, dgo, dbo, dy, x, g, mo, ro, N, C)
    torch.cuda.synchronize()
    assert max_rel_err(dinp.cpu(), torch.from_numpy(dxo + d0)) < 1e-4
    assert max_rel_err(dinp_b.float().cpu(), torch.from_numpy(dxo + d0)) < 1e-2
    assert max_rel_err(dg.cpu(), torch.from_numpy(dgo)) < 1e-4
    assert max_rel_err(db.cpu(), torch.from_numpy(dbo)) < 1e-4
    # fused column sums of the final dinp (the next linear layer's bias gradient)
    assert max_rel_err(dsum.cpu(), torch.from_numpy((dxo + d0).astype(np.float64).sum(0))) < 1e-4
    assert llmk.device_status() == 0


@pytest.mark.parametrize("C", [768, 1280, 200])
def test_layernorm_widths(cuda_dev, C):
    """Register-resident (C = 768, 1280) and generic (C = 200) LayerNorm paths vs the oracle."""
    import torch
    import llmk
    N = 257
    x = O.normal((N, C), 71, std=1.5)
    g = O.normal((C,), 72)
    be = O.normal((C,), 73)
    dy = O.normal((N, C), 74)
    s = llmk.stream_ptr()
    xd, gd, bd, dyd = T(x, cuda_dev), T(g, cuda_dev), T(be, cuda_dev), T(dy, cuda_dev)
    y = torch.empty(N, C, device=cuda_dev)
    mean = torch.empty(N, device=cuda_dev)
    rstd = torch.empty(N, device=cuda_dev)
    llmk.call("llmk_layernorm_forward", y.data_ptr(), llmk.F32, mean.data_ptr(), rstd.data_ptr(), xd.data_ptr(),
              gd.data_ptr(), bd.data_ptr(), N, C, s)
    dinp = torch.empty(N, C, device=cuda_dev)
    dg = torch.empty(C, device=cuda_dev)
    db = torch.empty(C, device=cuda_dev)
    ws_b = llmk.lib().llmk_layernorm_backward_workspace(N, C)
    ws = torch.empty(ws_b // 4 + 64, device=cuda_dev)
    llmk.call("llmk_layernorm_backward", dinp.data_ptr(), None, dg.data_ptr(), db.data_ptr(), None, dyd.data_ptr(),
              llmk.F32, xd.data_ptr(), gd.data_ptr(), mean.data_ptr(), rstd.data_ptr(), N, C, 0, ws.data_ptr(), ws_b,
              s)
    yo, mo, ro = np.zeros_like(x), np.zeros(N, np.float32), np.zeros(N, np.float32)
    O.orc().orc_layernorm_forward(yo, mo.ctypes.data, ro.ctypes.data, x, g, be, N, C)
    dxo, dgo, dbo = np.zeros_like(x), np.zeros(C, np.float32), np.zeros(C, np.float32)
    O.orc().orc_layernorm_backward(dxo, dgo, dbo, dy, x, g, mo, ro, N, C)
    torch.cuda.synchronize()
    assert max_rel_err(y, yo) < 1e-5
    assert max_rel_err(dinp, dxo) < 1e-4
    assert max_rel_err(dg, dgo) < 1e-4 and max_rel_err(db, dbo) < 1e-4


def test_gelu_residual_vs_oracle(cuda_dev):
    import torch
    import llmk
    n = 4096 * 3
    x = O.normal((n,), 21, std=2.0)
    dy = O.normal((n,), 22)
    s = llmk.stream_ptr()
    xd, dyd = T(x, cuda_dev), T(dy, cuda_dev)
    y = torch.empty(n, device=cuda_dev)
    llmk.call("llmk_gelu_forward", y.data_ptr(), xd.data_ptr(), llmk.F32, n, s)
    d = torch.empty(n, device=cuda_dev)
    llmk.call("llmk_gelu_backward", d.data_ptr(), dyd.data_ptr(), xd.data_ptr(), llmk.F32, n, 0, s)
    yo, do = np.zeros_like(x), np.zeros_like(x)
    O.orc().orc_gelu_forward(yo, x, n)
    O.orc().orc_gelu_backward(do, dy, x, n)
    torch.cuda.synchronize()
    assert max_rel_err(y.cpu(), torch.from_numpy(yo)) < 1e-5
    assert max_rel_err(d.cpu(), torch.from_numpy(do)) < 1e-5
    r = torch.empty(n, device=cuda_dev)
    llmk.call("llmk_residual_forward", r.data_ptr(), xd.data_ptr(), dyd.data_ptr(), llmk.F32, n, s)
    ro = np.zeros_like(x)
    O.orc().orc_residual_forward(ro, x, dy, n)
    torch.cuda.synchronize()
    assert torch.equal(r.cpu(), torch.from_numpy(ro))


def test_encoder_vs_oracle(cuda_dev):
    import torch
    import llmk
    B, Tt, C, V = 4, 64, 768, 50
    tok = O.tokens(B * Tt, V, 31)  # small vocabulary: many repeated tokens
    wte = O.normal((V, C), 32)
    wpe = O.normal((Tt, C), 33)
    dout = O.normal((B * Tt, C), 34)
    s = llmk.stream_ptr()
    out = torch.empty(B * Tt, C, device=cuda_dev)
    tokd = T(tok, cuda_dev)
    wted, wped = T(wte, cuda_dev), T(wpe, cuda_dev)  # keep the device copies alive until the kernel ran
    llmk.call("llmk_encoder_forward", out.data_ptr(), tokd.data_ptr(), wted.data_ptr(), wped.data_ptr(), B, Tt, C, s)
    oo = np.zeros((B * Tt, C), np.float32)
    O.orc().orc_encoder_forward(oo, tok, wte, wpe, B, Tt, C)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), torch.from_numpy(oo))
    dwte = T(np.zeros((V, C), np.float32), cuda_dev)
    dwpe = T(np.zeros((Tt, C), np.float32), cuda_dev)
    ws_b = llmk.lib().llmk_encoder_backward_workspace(B, Tt)
    ws = torch.empty(ws_b // 4 + 16, device=cuda_dev)
    doutd = T(dout, cuda_dev)
    llmk.call("llmk_encoder_backward", dwte.data_ptr(), dwpe.data_ptr(), doutd.data_ptr(), tokd.data_ptr(), B, Tt, C,
              V, ws.data_ptr(), ws_b, s)
    a, b = np.zeros((V, C), np.float32), np.zeros((Tt, C), np.float32)
    O.orc().orc_encoder_backward(a, b, dout, tok, B, Tt, C)
    torch.cuda.synchronize()
    assert max_rel_err(dwte.cpu(), torch.from_numpy(a)) < 1e-5
    assert max_rel_err(dwpe.cpu(), torch.from_numpy(b)) < 1e-5


@pytest.mark.parametrize("B,Tt,V", [(16, 1024, 50257), (5, 1000, 3000), (16, 1024, 70000), (20, 1000, 50257),
                                    (33, 1024, 3000)])
def test_encoder_backward_sizes(cuda_dev, B, Tt, V):
    """Sort paths: B*T = 16384 and 5000 with V < 2^16 (the one-CTA radix sort), 16384 with V = 70000 (the
    bitonic network, 16 keys per thread in registers), 20000 (the shared-memory network, padded to 32768);
    B*T = 33792 takes the scan fallback. dwte starts at zero, so the device's per-token sums in position
    order must equal the oracle's sequential accumulation bit for bit."""
    import torch
    import llmk
    C = 128
    tok = O.tokens(B * Tt, V, 35)
    dout = O.normal((B * Tt, C), 36)
    tokd, doutd = T(tok, cuda_dev), T(dout, cuda_dev)
    dwte = torch.zeros(V, C, device=cuda_dev)
    dwpe = torch.zeros(Tt, C, device=cuda_dev)
    ws_b = llmk.lib().llmk_encoder_backward_workspace(B, Tt)
    ws = torch.empty(ws_b // 4 + 16, device=cuda_dev)
    llmk.call("llmk_encoder_backward", dwte.data_ptr(), dwpe.data_ptr(), doutd.data_ptr(), tokd.data_ptr(), B, Tt, C,
              V, ws.data_ptr(), ws_b, llmk.stream_ptr())
    a, b = np.zeros((V, C), np.float32), np.zeros((Tt, C), np.float32)
    O.orc().orc_encoder_backward(a, b, dout, tok, B, Tt, C)
    torch.cuda.synchronize()
    assert max_rel_err(dwte, a) < 1e-5
    assert max_rel_err(dwpe, b) < 1e-5
    assert np.array_equal(dwte.cpu().numpy(), a)


@pytest.mark.parametrize("B,Tt", [(16, 1024), (20, 1000)])
def test_encoder_backward_frequent_tokens(cuda_dev, B, Tt):
    """Text-like token counts: a few tokens take most positions (runs of thousands in the sorted order), as
    frequent words do. Runs of up to 64 positions are summed in position order (bit-exact to the oracle's
    sequential accumulation); longer runs in 32 ordered segments: within fp32 rounding of the oracle, and
    the same bits on every call."""
    import torch
    import llmk
    C, V = 768, 50257
    rng = np.random.default_rng(37)
    tok = rng.integers(0, V, B * Tt).astype(np.int32)
    hot = rng.random(B * Tt)
    tok[hot < 0.30] = 11
    tok[(hot >= 0.30) & (hot < 0.45)] = 13
    tok[(hot >= 0.45) & (hot < 0.50)] = 50256
    dout = O.normal((B * Tt, C), 38)
    tokd, doutd = T(tok, cuda_dev), T(dout, cuda_dev)
    dwte = torch.zeros(V, C, device=cuda_dev)
    dwpe = torch.zeros(Tt, C, device=cuda_dev)
    ws_b = llmk.lib().llmk_encoder_backward_workspace(B, Tt)
    ws = torch.empty(ws_b // 4 + 16, device=cuda_dev)
    llmk.call("llmk_encoder_backward", dwte.data_ptr(), dwpe.data_ptr(), doutd.data_ptr(), tokd.data_ptr(), B, Tt, C,
              V, ws.data_ptr(), ws_b, llmk.stream_ptr())
    a, b = np.zeros((V, C), np.float32), np.zeros((Tt, C), np.float32)
    O.orc().orc_encoder_backward(a, b, dout, tok, B, Tt, C)
    torch.cuda.synchronize()
    got = dwte.cpu().numpy()
    counts = np.bincount(tok, minlength=V)
    short = counts <= 64
    assert np.array_equal(got[short], a[short])
    assert max_rel_err(dwte, a) < 1e-5
    assert max_rel_err(dwpe, b) < 1e-5
    # deterministic: a second call on zeroed gradients gives the same bits
    dwte2 = torch.zeros(V, C, device=cuda_dev)
    dwpe.zero_()
    llmk.call("llmk_encoder_backward", dwte2.data_ptr(), dwpe.data_ptr(), doutd.data_ptr(), tokd.data_ptr(), B, Tt, C,
              V, ws.data_ptr(), ws_b, llmk.stream_ptr())
    torch.cuda.synchronize()
    assert torch.equal(dwte2, dwte)


@pytest.mark.parametrize("dtname", ["f32", "bf16"])
def test_softmax_crossentropy_vs_oracle(cuda_dev, dtname):
    import torch
    import llmk
    BT, V, Vp = 64, 50257, 50304
    logits = O.normal((BT, Vp), 41, std=3.0)
    logits[:, V:] = 0.0
    tgt = O.tokens(BT, V, 42)
    dt = torch.float32 if dtname == "f32" else torch.bfloat16
    if dtname == "bf16":
        logits = bf(logits)
    s = llmk.stream_ptr()
    ld = T(logits, cuda_dev, dt)
    losses = torch.empty(BT, device=cuda_dev)
    dl = torch.empty(BT, Vp, device=cuda_dev, dtype=dt)
    tgtd = T(tgt, cuda_dev)
    llmk.call("llmk_softmax_crossentropy", losses.data_ptr(), dl.data_ptr(), ld.data_ptr(), llmk.dtype_code(ld),
              tgtd.data_ptr(), BT, V, Vp, 1.0 / BT, s)
    mean = torch.empty(1, device=cuda_dev)
    llmk.call("llmk_mean", mean.data_ptr(), losses.data_ptr(), BT, s)
    probs = np.zeros((BT, V), np.float32)
    O.orc().orc_softmax(probs, logits, BT, V, Vp)
    lo = np.zeros(BT, np.float32)
    mo = O.orc().orc_cross_entropy(lo.ctypes.data, probs, tgt, BT, V)
    dlo = np.zeros((BT, Vp), np.float32)
    O.orc().orc_cross_entropy_softmax_backward(dlo, probs, tgt, BT, V, Vp)
    torch.cuda.synchronize()
    assert max_rel_err(losses.cpu(), torch.from_numpy(lo)) < 1e-4
    assert abs(mean.item() - mo) / mo < 1e-5
    tol = 1e-4 if dtname == "f32" else 1e-2
    assert max_rel_err(dl.float().cpu(), torch.from_numpy(dlo)) < tol
    assert torch.count_nonzero(dl[:, V:]).item() == 0


@pytest.mark.parametrize("BT,V,Vp", [(400, 50257, 50304), (333, 1001, 1008)])
def test_softmax_crossentropy_rows_in_place(cuda_dev, BT, V, Vp):
    """bf16 rows streamed through shared memory: more rows than SMs (each CTA
    walks several rows through both buffers) and dlogits written over logits."""
    import torch
    import llmk
    logits = bf(O.normal((BT, Vp), 43, std=2.0))
    logits[:, V:] = 0.0
    tgt = O.tokens(BT, V, 44)
    ld = T(logits, cuda_dev, torch.bfloat16)
    losses = torch.empty(BT, device=cuda_dev)
    llmk.call("llmk_softmax_crossentropy", losses.data_ptr(), ld.data_ptr(), ld.data_ptr(), llmk.BF16,
              T(tgt, cuda_dev).data_ptr(), BT, V, Vp, 1.0 / BT, llmk.stream_ptr())
    probs = np.zeros((BT, V), np.float32)
    O.orc().orc_softmax(probs, logits, BT, V, Vp)
    lo = np.zeros(BT, np.float32)
    O.orc().orc_cross_entropy(lo.ctypes.data, probs, tgt, BT, V)
    dlo = np.zeros((BT, Vp), np.float32)
    O.orc().orc_cross_entropy_softmax_backward(dlo, probs, tgt, BT, V, Vp)
    torch.cuda.synchronize()
    assert llmk.device_status() == 0
    assert max_rel_err(losses.cpu(), torch.from_numpy(lo)) < 1e-4
    assert max_rel_err(ld.float().cpu(), torch.from_numpy(dlo)) < 1e-2
    assert torch.count_nonzero(ld[:, V:]).item() == 0


def test_adamw_vs_oracle(cuda_dev):
    import torch
    import llmk
    n = 1 << 16
    p0 = O.normal((n,), 51)
    s = llmk.stream_ptr()
    p = T(p0, cuda_dev)
    pb = torch.empty(n, device=cuda_dev, dtype=torch.bfloat16)
    m = torch.zeros(n, device=cuda_dev)
    v = torch.zeros(n, device=cuda_dev)
    po, mo, vo = p0.copy(), np.zeros(n, np.float32), np.zeros(n, np.float32)
    import ctypes
    hp = torch.empty(8, device=cuda_dev)
    for t in range(1, 6):
        g = O.normal((n,), 60 + t)
        gd = T(g, cuda_dev)
        if t % 2:
            llmk.call("llmk_adamw", p.data_ptr(), pb.data_ptr(), gd.data_ptr(), m.data_ptr(), v.data_ptr(), n, 3e-4,
                      0.9, 0.999, 1e-8, 0.01, t, 1.0, s)
        else:  # the same update with the hyperparameters read from device memory
            h8 = (ctypes.c_float * 8)()
            llmk.lib().llmk_adamw_hparams(h8, 3e-4, 0.9, 0.999, 1e-8, 0.01, t, 1.0)
            hp.copy_(torch.tensor(list(h8), dtype=torch.float32))
            llmk.call("llmk_adamw_device_hparams", p.data_ptr(), pb.data_ptr(), gd.data_ptr(), m.data_ptr(),
                      v.data_ptr(), n, hp.data_ptr(), s)
        O.orc().orc_adamw(po, g, mo, vo, n, 3e-4, 0.9, 0.999, 1e-8, 0.01, t)
    torch.cuda.synchronize()
    assert max_rel_err(p.cpu(), torch.from_numpy(po)) < 1e-5
    assert max_rel_err(pb.float().cpu(), torch.from_numpy(po)) < 1e-2
    assert max_rel_err(m.cpu(), torch.from_numpy(mo)) < 1e-5
