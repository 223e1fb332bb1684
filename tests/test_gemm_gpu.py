"""tcgen05 GEMM (llmk_gemm) against a plain PyTorch fp32 reference.

BF16 mode: the kernel and the reference see the same bf16-rounded operands,
so only accumulation order differs (tolerance 1e-4 max-rel). TF32 mode: the
reference multiplies the fp32 operands exactly, the kernel in tf32 (the
hot-path tolerance, 2e-3 max-rel).
"""
import pytest

from conftest import max_rel_err

pytestmark = pytest.mark.gpu

FORMS = [(0, 0), (0, 1), (1, 1), (1, 0)]  # (a_trans, b_trans): fwd, dinp, dweight, (A M-major, B K-major)


def _operands(torch, M, N, K, a_trans, b_trans, math, dev, seed):
    import llmk
    g = torch.Generator(device="cpu").manual_seed(seed)
    A = torch.randn(M, K, generator=g)
    B = torch.randn(N, K, generator=g)
    if math == llmk.MATH_BF16:
        A = A.bfloat16()
        B = B.bfloat16()
    A_st = (A.t() if a_trans else A).contiguous().to(dev)
    B_st = (B.t() if b_trans else B).contiguous().to(dev)
    ref = A.double() @ B.double().t()
    return A_st, B_st, ref


@pytest.mark.parametrize("form", FORMS)
@pytest.mark.parametrize("mathname", ["bf16", "tf32"])
# M < 256: single-CTA tiles; M >= 256: CTA-pair tiles of 256 rows, including a
# ragged last pair (640, 1000) and N / K that are not tile multiples
@pytest.mark.parametrize("shape", [(128, 256, 64), (256, 128, 128), (384, 768, 192), (200, 136, 72),
                                   (640, 392, 200), (1000, 520, 136)])
def test_gemm_forms(cuda_dev, form, mathname, shape):
    import torch
    import llmk
    math = llmk.MATH_BF16 if mathname == "bf16" else llmk.MATH_TF32
    M, N, K = shape
    a_trans, b_trans = form
    A, B, ref = _operands(torch, M, N, K, a_trans, b_trans, math, cuda_dev, seed=M * 7 + N + K)
    D = torch.full((M, N), float("nan"), device=cuda_dev)
    llmk.gemm(D, A, B, a_trans=a_trans, b_trans=b_trans, math=math, M=M, N=N, K=K)
    torch.cuda.synchronize()
    tol = 1e-4 if math == llmk.MATH_BF16 else 2e-3
    err = max_rel_err(D.cpu(), ref)
    assert err < tol, f"form={form} {mathname} shape={shape} max_rel={err:.3e}"
    assert llmk.device_status() == 0


@pytest.mark.parametrize("mathname", ["bf16", "tf32"])
def test_gemm_layer_shapes(cuda_dev, mathname):
    """GPT-2 124M shapes at BT=2048: fwd / dinp / dweight forms (dweight split-K)."""
    import torch
    import llmk
    math = llmk.MATH_BF16 if mathname == "bf16" else llmk.MATH_TF32
    tol = 1e-4 if math == llmk.MATH_BF16 else 2e-3
    BT = 2048
    for C_, OC in [(768, 2304), (768, 768), (768, 3072), (3072, 768)]:
        for (M, N, K, a_t, b_t) in [(BT, OC, C_, 0, 0), (BT, C_, OC, 0, 1), (OC, C_, BT, 1, 1)]:
            A, B, ref = _operands(torch, M, N, K, a_t, b_t, math, cuda_dev, seed=OC + K)
            ws_bytes = llmk.lib().llmk_gemm_workspace(M, N, K, math)
            ws = torch.empty(max(ws_bytes // 4, 1), device=cuda_dev)
            D = torch.full((M, N), float("nan"), device=cuda_dev)
            llmk.gemm(D, A, B, a_trans=a_t, b_trans=b_t, math=math, M=M, N=N, K=K, workspace=ws)
            torch.cuda.synchronize()
            err = max_rel_err(D.cpu(), ref)
            assert err < tol, f"{mathname} M={M} N={N} K={K} trans=({a_t},{b_t}) ws={ws_bytes} max_rel={err:.3e}"
    assert llmk.device_status() == 0


def test_gemm_weight_gradient_long_k(cuda_dev):
    """Weight-gradient form with K = 8192 tokens: 256-wide CTA-pair tiles and
    split-K sized to one wave (the planner's long-K path), bf16 and tf32."""
    import torch
    import llmk
    for math, tol in ((llmk.MATH_BF16, 1e-4), (llmk.MATH_TF32, 2e-3)):
        for M, N in ((768, 768), (2304, 768), (768, 3072)):
            K = 8192
            A, B, ref = _operands(torch, M, N, K, 1, 1, math, cuda_dev, seed=M + N)
            ws_bytes = llmk.lib().llmk_gemm_workspace(M, N, K, math)
            assert ws_bytes > 0  # split-K
            ws = torch.empty(ws_bytes // 4, device=cuda_dev)
            D = torch.full((M, N), float("nan"), device=cuda_dev)
            llmk.gemm(D, A, B, a_trans=1, b_trans=1, math=math, M=M, N=N, K=K, workspace=ws)
            torch.cuda.synchronize()
            err = max_rel_err(D.cpu(), ref)
            assert err < tol, (math, M, N, err)
    assert llmk.device_status() == 0


@pytest.mark.parametrize("M", [192, 512])
def test_gemm_epilogues(cuda_dev, M):
    """bias, residual, GELU (+ pre-activation store), GELU-backward, accumulate, bf16 output
    (M = 192: single-CTA tiles, 512: CTA pairs)."""
    import torch
    import llmk
    N, K = 512, 128
    A, B, ref = _operands(torch, M, N, K, 0, 0, llmk.MATH_BF16, cuda_dev, seed=5)
    ref = ref.float()
    bias = torch.randn(N, device=cuda_dev)
    res = torch.randn(M, N, device=cuda_dev)
    # bias + residual, fp32 out
    D = torch.empty(M, N, device=cuda_dev)
    llmk.gemm(D, A, B, bias=bias, residual=res)
    exp = ref.to(cuda_dev) + bias + res
    assert max_rel_err(D, exp) < 1e-4
    # accumulate
    D0 = torch.randn(M, N, device=cuda_dev)
    D = D0.clone()
    llmk.gemm(D, A, B, flags=llmk.EPI_ACCUMULATE)
    assert max_rel_err(D, D0 + ref.to(cuda_dev)) < 1e-4
    # GELU with pre-activation store, bf16 out
    Dg = torch.empty(M, N, device=cuda_dev, dtype=torch.bfloat16)
    pre = torch.empty(M, N, device=cuda_dev, dtype=torch.bfloat16)
    llmk.gemm(Dg, A, B, bias=bias, aux=pre, flags=llmk.EPI_GELU)
    z = ref.to(cuda_dev) + bias
    assert max_rel_err(pre.float(), z) < 1e-2
    gelu = torch.nn.functional.gelu(z, approximate="tanh")
    assert max_rel_err(Dg.float(), gelu) < 1e-2
    # fp32 output with a bf16 pre-activation (stored directly, not by TMA)
    Df = torch.empty(M, N, device=cuda_dev)
    pre2 = torch.empty(M, N, device=cuda_dev, dtype=torch.bfloat16)
    llmk.gemm(Df, A, B, bias=bias, aux=pre2, flags=llmk.EPI_GELU)
    assert max_rel_err(pre2.float(), z) < 1e-2
    assert max_rel_err(Df, gelu) < 1e-4
    # GELU backward: D = (A B^T) * gelu'(pre)
    Db = torch.empty(M, N, device=cuda_dev, dtype=torch.bfloat16)
    llmk.gemm(Db, A, B, aux=pre, flags=llmk.EPI_GELU_BWD)
    x = pre.float().requires_grad_(True)
    torch.nn.functional.gelu(x, approximate="tanh").backward(ref.to(cuda_dev))
    assert max_rel_err(Db.float(), x.grad) < 1e-2
    torch.cuda.synchronize()
    assert llmk.device_status() == 0


@pytest.mark.parametrize("M,N,K", [(600, 776, 192), (1000, 200, 136), (512, 3072, 768)])
def test_gemm_operand_epilogues_ragged(cuda_dev, M, N, K):
    """The two epilogue programs that take a per-element operand by TMA tile loads, on CTA-pair tiles with a
    ragged last row block and column block (the operand's edge chunks load as zeros, D's edge stores are
    clipped): bias + fp32 residual with a row stride wider than N (the residual GEMMs; K <= 1024 and
    longer), and GELU-backward with B N-major and bf16 D / pre-activation (the FC-projection input
    gradient)."""
    import torch
    import llmk
    A, B, ref = _operands(torch, M, N, K, 0, 0, llmk.MATH_BF16, cuda_dev, seed=11)
    ref = ref.float().to(cuda_dev)
    g = torch.Generator(device="cpu").manual_seed(12)
    bias = torch.randn(N, generator=g).to(cuda_dev)
    res_full = torch.randn(M, N + 8, generator=g).to(cuda_dev)
    res = res_full[:, :N]
    D = torch.full((M, N), float("nan"), device=cuda_dev)
    llmk.gemm(D, A, B, bias=bias, residual=res)
    assert max_rel_err(D, ref + bias + res) < 1e-4
    # GELU backward, B stored [K][N] (N-major) as the input-gradient GEMMs keep it
    Bt = B.t().contiguous()
    pre = (torch.randn(M, N, generator=g) * 2).bfloat16().to(cuda_dev)
    Db = torch.full((M, N), float("nan"), device=cuda_dev, dtype=torch.bfloat16)
    llmk.gemm(Db, A, Bt, b_trans=True, aux=pre, flags=llmk.EPI_GELU_BWD)
    x = pre.float().requires_grad_(True)
    torch.nn.functional.gelu(x, approximate="tanh").backward(ref)
    assert max_rel_err(Db.float(), x.grad) < 1e-2
    torch.cuda.synchronize()
    assert llmk.device_status() == 0


def test_gemm_rejects_misaligned(cuda_dev):
    import torch
    import llmk
    A = torch.randn(64, 20, device=cuda_dev).bfloat16()  # 40-byte rows
    B = torch.randn(64, 20, device=cuda_dev).bfloat16()
    D = torch.empty(64, 64, device=cuda_dev)
    with pytest.raises(llmk.LlmkError) as e:
        llmk.gemm(D, A, B)
    assert e.value.code == 2
