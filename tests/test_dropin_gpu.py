"""The drop-in boundary, exercised with data: the reference's OWN CUDA trainer
(gpt2cuda::GPT2 and gpt2cuda::Layer from gpt2/cuda/gpt2cuda.cu and layer.cu,
compiled unchanged from the reference tree) linked against
llm.cpp_b200/dropin/gpt2cuda_llmk.cu and libllmk.so in place of the
reference's op sources (oracle/_ref/libgpt2cuda_llmk.so, built by
`make -C oracle dropin` where the reference tree exists; skipped without it).

- 20 training steps of configuration 0 (GPT-2 124M, B=4, T=64, seed 1337,
  AdamW lr 3e-4, one fixed batch) through the reference's Forward / ZeroGrad /
  Backward / Update: every step's loss within 0.5% of the reference's CPU
  losses (the precision is the reference GPU path's: TF32 GEMMs, fp16
  attention operands).
- The reference's host-pointer test entry points (matmul.cuh:10,16,
  attention.cuh:6-7) against the oracle: TF32 GEMM bar 2e-3, attention 1e-2
  (fp16 operands, the reference's own attention test tolerance,
  tests/gpt2/cuda/test_cuda_attention.cpp:565-666).
"""
import ctypes as C
import json
import os

import numpy as np
import pytest

import oracle as O
from conftest import max_rel_err

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(os.path.dirname(HERE), "oracle", "_ref", "libgpt2cuda_llmk.so")
fp = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
ip = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def _lib():
    if not os.path.exists(LIB):
        pytest.skip("oracle/_ref/libgpt2cuda_llmk.so not built (needs the reference tree: make -C oracle dropin)")
    L = C.CDLL(LIB)
    L.gpt2cuda_harness_error.restype = C.c_char_p
    L.gpt2cuda_harness_train.argtypes = [C.c_char_p, C.c_int, C.c_int, ip, ip, C.c_int, C.c_float, fp]
    L.gpt2cuda_harness_matmul_host.argtypes = [fp, fp, fp, C.c_void_p, fp, fp, fp, C.c_void_p] + [C.c_int] * 4
    L.gpt2cuda_harness_attention_host.argtypes = [fp, fp, fp, fp, fp] + [C.c_int] * 4
    return L


def test_reference_trainer_on_llmk_config0(cuda_dev, tmp_path):
    L = _lib()
    fx = json.load(open(os.path.join(HERE, "golden", "gpt2_124m_b4t64_losses.json")))
    cfg = O.config()
    B, T, steps = fx["B"], fx["T"], fx["steps"]
    params = O.init_params(cfg, fx["seed"])
    toks = O.tokens(B * T + 1, cfg.vocab_size, fx["seed"])
    ck = str(tmp_path / "gpt2_124m.bin")
    O.write_checkpoint(ck, cfg, params)
    losses = np.zeros(steps, np.float32)
    rc = L.gpt2cuda_harness_train(ck.encode(), B, T, toks[:-1].copy(), toks[1:].copy(), steps, fx["lr"], losses)
    assert rc == 0, L.gpt2cuda_harness_error()
    rel = [abs(a - b) / b for a, b in zip(losses.tolist(), fx["losses"])]
    print("reference gpt2cuda::GPT2 on llmk", [round(float(x), 4) for x in losses])
    print("rel", [f"{x:.2e}" for x in rel])
    assert max(rel) <= 5e-3, rel


def test_reference_host_pointer_ops_vs_oracle(cuda_dev):
    L = _lib()
    B, T, C_, Oc = 2, 128, 768, 2304
    x = O.normal((B * T, C_), 61)
    W = O.normal((Oc, C_), 62)
    b = O.normal((Oc,), 63)
    dout = O.normal((B * T, Oc), 64)
    out = np.zeros((B * T, Oc), np.float32)
    dinp = O.normal((B * T, C_), 65)  # the reference accumulates dinp and dW
    dW = O.normal((Oc, C_), 66)
    db = np.zeros(Oc, np.float32)
    di_ref, dW_ref = dinp.copy(), dW.copy()
    rc = L.gpt2cuda_harness_matmul_host(out, dinp, dW, db.ctypes.data, dout, x, W, b.ctypes.data, B, T, C_, Oc)
    assert rc == 0, L.gpt2cuda_harness_error()
    y_ref = np.zeros_like(out)
    O.orc().orc_matmul_forward(y_ref, x, W, b.ctypes.data, B * T, C_, Oc)
    db_ref = np.zeros(Oc, np.float32)
    O.orc().orc_matmul_backward(di_ref, dW_ref, db_ref.ctypes.data, dout, x, W, B * T, C_, Oc)
    for name, a, r in (("out", out, y_ref), ("dinp", dinp, di_ref), ("dW", dW, dW_ref), ("dbias", db, db_ref)):
        assert max_rel_err(a, r) < 2e-3, name
    # causal attention, head size 64
    NH, T2 = 4, 256
    qkv = O.normal((B, T2, 3 * 64 * NH), 67)
    do = O.normal((B, T2, 64 * NH), 68)
    o = np.zeros((B, T2, 64 * NH), np.float32)
    lse = np.zeros((B, NH, T2), np.float32)
    dqkv = np.zeros_like(qkv)
    rc = L.gpt2cuda_harness_attention_host(o, lse, dqkv, do, qkv, B, T2, 3 * 64 * NH, NH)
    assert rc == 0, L.gpt2cuda_harness_error()
    C2 = 64 * NH
    o_ref = np.zeros_like(o)
    att = np.zeros((B, NH, T2, T2), np.float32)
    lse_ref = np.zeros((B, NH, T2), np.float32)
    O.orc().orc_attention_forward(o_ref, att, lse_ref.ctypes.data, qkv, B, T2, C2, NH)
    dqkv_ref = np.zeros_like(qkv)
    O.orc().orc_attention_backward(dqkv_ref, do, qkv, att, B, T2, C2, NH)
    assert max_rel_err(o, o_ref) < 1e-2
    assert max_rel_err(lse, lse_ref) < 1e-2
    assert max_rel_err(dqkv, dqkv_ref) < 1e-2
