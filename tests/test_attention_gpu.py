"""tcgen05 causal flash attention vs the oracle (reference CPU algorithm).

Inputs are seeded N(0,1) from the oracle's generator, rounded to the 16-bit
operand type for the device; the oracle consumes the same rounded values in
fp32. Tolerance: max relative error 1e-2 (the BF16 bar of the hot path) on O,
LSE, dQ, dK, dV with bf16 operands; 3e-3 with fp16 operands (the operand
type of the TF32 training mode: 3 more mantissa bits in Q, K, V, P, dO, dS).
"""
import numpy as np
import pytest

import oracle as O
from conftest import max_rel_err

pytestmark = pytest.mark.gpu


def _bf16_round(x):
    import torch
    return torch.from_numpy(x).bfloat16().float().numpy()


def _round(x, op):
    import torch
    t = torch.from_numpy(x)
    return (t.half() if op == "f16" else t.bfloat16()).float().numpy()


TOL = {"bf16": 1e-2, "f16": 3e-3}


def _run_gpu(qkv_np, dout_np, B, T, C, NH, dev, io="bf16", op="bf16"):
    """One forward + backward through the C ABI. op: operand type of qkv
    ("bf16" / "f16"); io: dtype of O, dO and dqkv ("f32" or the operand type)."""
    import torch
    import llmk
    odt, ocode = (torch.float16, llmk.F16) if op == "f16" else (torch.bfloat16, llmk.BF16)
    tdt, code = (odt, ocode) if io != "f32" else (torch.float32, llmk.F32)
    qkv = torch.from_numpy(qkv_np).to(dev).to(odt).contiguous()
    dout = torch.from_numpy(dout_np).to(dev).to(tdt).contiguous()
    out = torch.full((B, T, C), float("nan"), device=dev, dtype=tdt)
    lse = torch.full((B, NH, T), float("nan"), device=dev)
    s = llmk.stream_ptr()
    llmk.call("llmk_attention_forward", out.data_ptr(), code, lse.data_ptr(), qkv.data_ptr(), ocode, B, T, 3 * C, NH,
              s)
    ws_b = llmk.lib().llmk_attention_backward_workspace(B, T, 3 * C, NH)
    ws = torch.empty(ws_b // 4 + 64, device=dev)
    dqkv = torch.full((B, T, 3 * C), float("nan"), device=dev, dtype=tdt)
    llmk.call("llmk_attention_backward", dqkv.data_ptr(), dout.data_ptr(), out.data_ptr(), code, qkv.data_ptr(), ocode,
              lse.data_ptr(), B, T, 3 * C, NH, ws.data_ptr(), ws_b, s)
    torch.cuda.synchronize()
    assert llmk.device_status() == 0
    return out.float().cpu().numpy(), lse.cpu().numpy(), dqkv.float().cpu().numpy()


@pytest.mark.parametrize("op,io", [("bf16", "bf16"), ("bf16", "f32"), ("f16", "f16"), ("f16", "f32")])
# (4, 600, 12): 120 pair items over at most 148 persistent CTAs with a ragged
# last tile; (1, 384, 2): an odd number of query tiles (a pair without B)
@pytest.mark.parametrize("B,T,NH", [(1, 128, 1), (2, 256, 2), (1, 200, 3), (2, 64, 2), (1, 384, 2), (1, 1, 1),
                                    (4, 600, 12)])
def test_attention_vs_oracle(cuda_dev, B, T, NH, op, io):
    C = 64 * NH
    qkv = _round(O.normal((B, T, 3 * C), 100 + T), op)
    dout = _round(O.normal((B, T, C), 200 + T), op)
    out_g, lse_g, dqkv_g = _run_gpu(qkv, dout, B, T, C, NH, cuda_dev, io, op)
    tol = TOL[op]
    out_o = np.zeros((B, T, C), np.float32)
    att = np.zeros((B, NH, T, T), np.float32)
    lse_o = np.zeros((B, NH, T), np.float32)
    O.orc().orc_attention_forward(out_o, att, lse_o.ctypes.data, O.f32a(qkv), B, T, C, NH)
    dqkv_o = np.zeros((B, T, 3 * C), np.float32)
    # the backward's dO.O uses the device's bf16 O, as the kernel does
    O.orc().orc_attention_backward(dqkv_o, O.f32a(dout), O.f32a(qkv), att, B, T, C, NH)
    assert max_rel_err(out_g, out_o) < tol, max_rel_err(out_g, out_o)
    assert max_rel_err(lse_g, lse_o) < tol
    # relative to the largest gradient entry of dQ|dK|dV: for T = 1 the true dQ
    # and dK are exactly zero (softmax over one key), so a per-part scale is empty
    scale = np.abs(dqkv_o).max()
    for name, sl in (("dq", slice(0, C)), ("dk", slice(C, 2 * C)), ("dv", slice(2 * C, 3 * C))):
        e = np.abs(dqkv_g[..., sl] - dqkv_o[..., sl]).max() / scale
        assert e < tol, f"{name} max_rel={e:.3e}"


def test_attention_config2_vs_torch(cuda_dev):
    """Config 2 shape (B=8, NH=12, T=1024, hd=64) against an fp32 PyTorch reference on the GPU."""
    import torch
    B, NH, T, C = 8, 12, 1024, 768
    qkv_np = O.normal((B, T, 3 * C), 7)
    dout_np = O.normal((B, T, C), 8)
    out_g, lse_g, dqkv_g = _run_gpu(qkv_np, dout_np, B, T, C, NH, cuda_dev)
    qkv = torch.from_numpy(qkv_np).to(cuda_dev).bfloat16().float().requires_grad_(True)
    q, k, v = qkv.split(C, dim=2)
    q = q.view(B, T, NH, 64).transpose(1, 2)
    k = k.view(B, T, NH, 64).transpose(1, 2)
    v = v.view(B, T, NH, 64).transpose(1, 2)
    s = (q @ k.transpose(-1, -2)) * 0.125
    mask = torch.ones(T, T, device=cuda_dev, dtype=torch.bool).tril()
    s = s.masked_fill(~mask, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    y = (torch.softmax(s, dim=-1) @ v).transpose(1, 2).reshape(B, T, C)
    y.backward(torch.from_numpy(dout_np).to(cuda_dev).bfloat16().float())
    assert max_rel_err(torch.from_numpy(out_g), y.detach().cpu()) < 1e-2
    assert max_rel_err(torch.from_numpy(lse_g), lse.detach().cpu()) < 1e-2
    g = qkv.grad.cpu()
    for name, sl in (("dq", slice(0, C)), ("dk", slice(C, 2 * C)), ("dv", slice(2 * C, 3 * C))):
        e = max_rel_err(torch.from_numpy(dqkv_g[..., sl]), g[..., sl])
        assert e < 1e-2, f"{name} max_rel={e:.3e}"


def test_attention_rejects_head_size(cuda_dev):
    import torch
    import llmk
    qkv = torch.zeros(1, 128, 3 * 96, device=cuda_dev, dtype=torch.bfloat16)
    out = torch.zeros(1, 128, 96, device=cuda_dev, dtype=torch.bfloat16)
    lse = torch.zeros(1, 3, 128, device=cuda_dev)
    with pytest.raises(llmk.LlmkError) as e:
        llmk.call("llmk_attention_forward", out.data_ptr(), llmk.BF16, lse.data_ptr(), qkv.data_ptr(), llmk.BF16, 1,
                  128, 288, 3, llmk.stream_ptr())
    assert e.value.code == 2


def test_attention_f32_output_is_unrounded(cuda_dev):
    """fp32 output mode returns the fp32 accumulator: it rounds to the bf16 output
    of the bf16 mode (same kernel, same q, k, v) and is not itself bf16-valued."""
    B, T, NH = 2, 256, 2
    C = 64 * NH
    qkv = _bf16_round(O.normal((B, T, 3 * C), 31))
    dout = _bf16_round(O.normal((B, T, C), 32))
    o16, l16, _ = _run_gpu(qkv, dout, B, T, C, NH, cuda_dev, "bf16")
    o32, l32, _ = _run_gpu(qkv, dout, B, T, C, NH, cuda_dev, "f32")
    assert np.array_equal(l16, l32)
    assert np.array_equal(_bf16_round(o32), o16)
    assert not np.array_equal(o32, o16)
