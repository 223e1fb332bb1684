"""Small, self-contained launches of single llmk kernels for profiling.

    python llm.cpp_b200/profile_case.py gemm    [M N K] [--trans A B] [--reps R]
    python llm.cpp_b200/profile_case.py attn    [B T NH] [--reps R]
    python llm.cpp_b200/profile_case.py attnbwd [B T NH] [--reps R]
    python llm.cpp_b200/profile_case.py step    [B T]    [--reps R]
    python llm.cpp_b200/profile_case.py gemmset [BT]     [--reps R]
    python llm.cpp_b200/profile_case.py lmxent  [BT]     [--variant fused|unfused|gemm] [--reps R]

lmxent runs the GPT-2 124M lm_head + softmax + cross-entropy (+ dlogits in
place) at BT tokens: fused (llmk_matmul_crossentropy_forward), unfused
(llmk_gemm + llmk_softmax_crossentropy) or the logits GEMM alone.

gemmset runs each GEMM shape of one GPT-2 124M training step at BT tokens
(fwd / dinp / dweight of QKV, attproj, FC, FCproj and the tied lm_head, in
that order, bf16) once per rep, for per-shape ncu counters.

Each case allocates its inputs once, runs one warm-up launch and R timed
launches, prints the CUDA-event time per launch, and exits 0. Sizes default
to shapes whose operands exceed the 126 MB L2 while holding only a few GB,
so an `ncu --set full -k <kernel> -c 1..3` capture of them ends quickly.
"""
from __future__ import annotations

import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["gemm", "attn", "attnbwd", "step", "gemmset", "lmxent"])
    ap.add_argument("--variant", choices=["fused", "unfused", "gemm"], default="fused")
    ap.add_argument("dims", nargs="*", type=int)
    ap.add_argument("--trans", nargs=2, type=int, default=[0, 0])
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--out-bf16", action="store_true")
    a = ap.parse_args()
    import torch
    import llmk
    torch.cuda.set_device(0)
    dev = "cuda"
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if a.case == "gemm":
        M, N, K = (a.dims + [16384, 4096, 768][len(a.dims):])[:3]
        at, bt = a.trans
        A = torch.randn((K, M) if at else (M, K), device=dev).bfloat16()
        B = torch.randn((K, N) if bt else (N, K), device=dev).bfloat16()
        D = torch.empty(M, N, device=dev, dtype=torch.bfloat16 if a.out_bf16 else torch.float32)
        wsb = llmk.lib().llmk_gemm_workspace(M, N, K, llmk.MATH_BF16)
        ws = torch.empty(max(wsb // 4, 1), device=dev)
        run = lambda: llmk.gemm(D, A, B, a_trans=at, b_trans=bt, M=M, N=N, K=K, workspace=ws)
        flop = 2.0 * M * N * K
    elif a.case == "attn":
        Bb, T, NH = (a.dims + [8, 1024, 12][len(a.dims):])[:3]
        C = 64 * NH
        qkv = torch.randn(Bb, T, 3 * C, device=dev).bfloat16()
        out = torch.empty(Bb, T, C, device=dev, dtype=torch.bfloat16)
        lse = torch.empty(Bb, NH, T, device=dev)
        s = llmk.stream_ptr()
        run = lambda: llmk.call("llmk_attention_forward", out.data_ptr(), llmk.BF16, lse.data_ptr(), qkv.data_ptr(),
                                llmk.BF16, Bb, T, 3 * C, NH, s)
        flop = 4.0 * Bb * NH * 64 * T * (T + 1) / 2
    elif a.case == "attnbwd":
        Bb, T, NH = (a.dims + [8, 1024, 12][len(a.dims):])[:3]
        C = 64 * NH
        s = llmk.stream_ptr()
        qkv = torch.randn(Bb, T, 3 * C, device=dev).bfloat16()
        out = torch.empty(Bb, T, C, device=dev, dtype=torch.bfloat16)
        dout = torch.randn(Bb, T, C, device=dev).bfloat16()
        dqkv = torch.empty(Bb, T, 3 * C, device=dev, dtype=torch.bfloat16)
        lse = torch.empty(Bb, NH, T, device=dev)
        wsb = llmk.lib().llmk_attention_backward_workspace(Bb, T, 3 * C, NH)
        ws = torch.empty(wsb // 4 + 64, device=dev)
        llmk.call("llmk_attention_forward", out.data_ptr(), llmk.BF16, lse.data_ptr(), qkv.data_ptr(), llmk.BF16, Bb, T,
                  3 * C, NH, s)
        run = lambda: llmk.call("llmk_attention_backward", dqkv.data_ptr(), dout.data_ptr(), out.data_ptr(), llmk.BF16,
                                qkv.data_ptr(), llmk.BF16, lse.data_ptr(), Bb, T, 3 * C, NH, ws.data_ptr(), wsb, s)
        # S = QK^T, dP = dO V^T, dV += P^T dO, dK += dS^T Q, dQ += dS K over the causal half
        flop = 10.0 * Bb * NH * 64 * T * (T + 1) / 2
    elif a.case == "gemmset":
        BT = (a.dims + [16384])[0]
        C, Vp = 768, 50304
        shapes = []
        for IC, OC in [(C, 3 * C), (C, C), (C, 4 * C), (4 * C, C)]:
            shapes += [(BT, OC, IC, 0, 0), (BT, IC, OC, 0, 1), (OC, IC, BT, 1, 1)]
        shapes += [(BT, Vp, C, 0, 0), (BT, C, Vp, 0, 1), (Vp, C, BT, 1, 1)]
        bufs = []
        for (M, N, K, at, bt) in shapes:
            A = torch.randn((K, M) if at else (M, K), device=dev).bfloat16()
            B = torch.randn((K, N) if bt else (N, K), device=dev).bfloat16()
            D = torch.empty(M, N, device=dev, dtype=torch.float32 if at else torch.bfloat16)
            wsb = llmk.lib().llmk_gemm_workspace(M, N, K, llmk.MATH_BF16)
            bufs.append((A, B, D, torch.empty(max(wsb // 4, 1), device=dev), M, N, K, at, bt))

        def run():
            for (A, B, D, ws, M, N, K, at, bt) in bufs:
                llmk.gemm(D, A, B, a_trans=at, b_trans=bt, M=M, N=N, K=K, workspace=ws)
        flop = sum(2.0 * M * N * K for (_, _, _, _, M, N, K, _, _) in bufs)
    elif a.case == "lmxent":
        BT = (a.dims + [16384])[0]
        C, V, Vp = 768, 50257, 50304
        s = llmk.stream_ptr()
        x = torch.randn(BT, C, device=dev).bfloat16()
        W = (torch.randn(Vp, C, device=dev) * 0.05).bfloat16()
        tg = torch.randint(0, V, (BT,), device=dev, dtype=torch.int32)
        logits = torch.empty(BT, Vp, device=dev, dtype=torch.bfloat16)
        losses = torch.empty(BT, device=dev)
        wsb = llmk.lib().llmk_matmul_softmax_workspace(BT, Vp)
        ws = torch.empty(wsb // 4 + 4, device=dev)
        if a.variant == "fused":
            run = lambda: llmk.call("llmk_matmul_crossentropy_forward", losses.data_ptr(), logits.data_ptr(),
                                    llmk.BF16, x.data_ptr(), W.data_ptr(), None, tg.data_ptr(), BT, C, Vp, V,
                                    1.0 / BT, 1, llmk.MATH_BF16, ws.data_ptr(), wsb, s)
        elif a.variant == "unfused":
            def run():
                llmk.gemm(logits, x, W)
                llmk.call("llmk_softmax_crossentropy", losses.data_ptr(), logits.data_ptr(), logits.data_ptr(),
                          llmk.BF16, tg.data_ptr(), BT, V, Vp, 1.0 / BT, s)
        else:
            run = lambda: llmk.gemm(logits, x, W)
        flop = 2.0 * BT * Vp * C
    else:
        Bb, T = (a.dims + [16, 1024][len(a.dims):])[:2]
        m = llmk.GPT2(Bb, T)
        import numpy as np
        n = m.n
        m.load_parameters((np.random.default_rng(0).standard_normal(n) * 0.02).astype(np.float32))
        toks = np.random.default_rng(1).integers(0, 50257, size=Bb * T + 1, dtype=np.int32)
        m.train_step(toks[:-1], toks[1:], 0.0, t=1, want_loss=False)
        d_in, d_tg = m.buffers()
        stream = torch.cuda.ExternalStream(m.stream)
        torch.cuda.set_stream(stream)
        state = {"t": 2}

        def run():
            m.step_device(d_in, d_tg, 3e-4, state["t"])
            state["t"] += 1
        flop = 0.0
    n0 = llmk.lib().llmk_launch_count()
    run()
    torch.cuda.synchronize()
    print(f"llmk launches before the timed region: {llmk.lib().llmk_launch_count()}, "
          f"per launch of the case: {llmk.lib().llmk_launch_count() - n0}")
    s = torch.cuda.current_stream()
    e0.record(s)
    for _ in range(a.reps):
        run()
    e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / a.reps
    extra = f", {flop / ms / 1e9:.1f} TFLOP/s" if flop else ""
    tag = f"{a.case}/{a.variant}" if a.case == "lmxent" else a.case
    print(f"{tag} {a.dims}: {ms:.4f} ms per launch{extra}; device status {llmk.device_status()}")


if __name__ == "__main__":
    main()
