"""Pins the oracle (oracle/oracle.c) to the reference's own golden vectors.

The vectors are the literal PyTorch outputs in the reference's CPU gtest
suite (tests/gpt2/test_*.cpp), extracted as text into
tests/golden/reference_unit_vectors.json. Each case uses the reference
test's own tolerance, with its metric: Eigen isApprox(a, b, p) is
||a - b|| <= p * min(||a||, ||b||).
"""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = json.load(open(os.path.join(HERE, "golden", "reference_unit_vectors.json")))


def is_approx(a, b, p):
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    return np.linalg.norm(a - b) <= p * min(np.linalg.norm(a), np.linalg.norm(b))


def g(case, name, shape=None):
    v = np.array(GOLD[case][name], dtype=np.float32)
    return v.reshape(shape) if shape else v


@pytest.fixture(scope="module")
def O():
    import oracle  # oracle/oracle.py (tests put the repo root on sys.path)
    return oracle


def test_matmul_forward(O):
    c = "test_matmul.cpp::forward1"
    x = g(c, "inputs", (2, 3, 4))
    w_cpu = g(c, "matmul.weight", (4, 5))  # Eigen (C, OC)
    W = np.ascontiguousarray(w_cpu.T)      # (OC, C)
    b = g(c, "matmul.bias")
    out = np.zeros((6, 5), np.float32)
    O.orc().orc_matmul_forward(out, O.f32a(x.reshape(6, 4)), O.f32a(W), b.ctypes.data, 6, 4, 5)
    exp = g(c, "resexp", (2, 3, 5)).reshape(6, 5)
    for bb in range(2):
        assert is_approx(out[3 * bb:3 * bb + 3], exp[3 * bb:3 * bb + 3], 1e-3)


def test_matmul_backward(O):
    c = "test_matmul.cpp::backward1"
    x = np.concatenate([g(c, "inputs[0]", (3, 4)), g(c, "inputs[1]", (3, 4))])
    W = O.f32a(g(c, "matmul.weight", (4, 5)).T)
    dout = np.ones((6, 5), np.float32)
    dinp = np.zeros((6, 4), np.float32)
    dW = np.zeros((5, 4), np.float32)
    db = np.zeros(5, np.float32)
    O.orc().orc_matmul_backward(dinp, dW, db.ctypes.data, dout, O.f32a(x), W, 6, 4, 5)
    exp = np.concatenate([g(c, "resexp[0]", (3, 4)), g(c, "resexp[1]", (3, 4))])
    assert is_approx(dinp[:3], exp[:3], 1e-3) and is_approx(dinp[3:], exp[3:], 1e-3)
    assert is_approx(dW.T, g(c, "d_weightexp", (4, 5)), 1e-3)
    assert is_approx(db, g(c, "d_biasexp"), 1e-3)


def _qkv(c):
    return np.concatenate([g(c, "inputs[0]", (1, 3, 12)), g(c, "inputs[1]", (1, 3, 12))])


def test_attention_forward(O):
    c = "test_attention.cpp::forward1"
    qkv = O.f32a(_qkv(c))
    out = np.zeros((2, 3, 4), np.float32)
    att = np.zeros((2, 2, 3, 3), np.float32)
    O.orc().orc_attention_forward(out, att, None, qkv, 2, 3, 4, 2)
    for b in range(2):
        assert is_approx(out[b], g(c, f"resexp[{b}]", (3, 4)), 1e-3)


def test_attention_backward(O):
    c = "test_attention.cpp::backward1"
    qkv = O.f32a(_qkv(c))
    out = np.zeros((2, 3, 4), np.float32)
    att = np.zeros((2, 2, 3, 3), np.float32)
    O.orc().orc_attention_forward(out, att, None, qkv, 2, 3, 4, 2)
    dqkv = np.zeros((2, 3, 12), np.float32)
    O.orc().orc_attention_backward(dqkv, np.ones((2, 3, 4), np.float32), qkv, att, 2, 3, 4, 2)
    for b in range(2):
        assert is_approx(dqkv[b], g(c, f"resexp[{b}]", (3, 12)), 1e-3)


@pytest.mark.parametrize("case", ["forward1", "forward2"])
def test_layernorm_forward(O, case):
    c = f"test_layernorm.cpp::{case}"
    x = g(c, "inputs", (6, 4))
    out = np.zeros((6, 4), np.float32)
    O.orc().orc_layernorm_forward(out, None, None, O.f32a(x), np.ones(4, np.float32), np.zeros(4, np.float32), 6, 4)
    exp = g(c, "resexp", (6, 4))
    assert is_approx(out[:3], exp[:3], 1e-3) and is_approx(out[3:], exp[3:], 1e-3)


@pytest.mark.parametrize("case", ["backward1", "backward2"])
def test_layernorm_backward(O, case):
    c = f"test_layernorm.cpp::{case}"
    gamma, beta = g(c, "layernorm.gamma"), g(c, "layernorm.beta")
    x = O.f32a(np.concatenate([g(c, "inputs[0]", (3, 4)), g(c, "inputs[1]", (3, 4))]))
    if case == "backward1":
        dout = np.ones((6, 4), np.float32)
    else:
        dout = O.f32a(np.concatenate([g(c, "d_outputs[0]", (3, 4)), g(c, "d_outputs[1]", (3, 4))]))
    out = np.zeros((6, 4), np.float32)
    mean = np.zeros(6, np.float32)
    rstd = np.zeros(6, np.float32)
    O.orc().orc_layernorm_forward(out, mean.ctypes.data, rstd.ctypes.data, x, gamma, beta, 6, 4)
    dinp = np.zeros((6, 4), np.float32)
    dg = np.zeros(4, np.float32)
    db = np.zeros(4, np.float32)
    O.orc().orc_layernorm_backward(dinp, dg, db, dout, x, gamma, mean, rstd, 6, 4)
    for b in range(2):
        assert is_approx(dinp[3 * b:3 * b + 3], g(c, f"resexp[{b}]", (3, 4)), 5e-3)
    assert is_approx(dg, g(c, "d_gamma_exp"), 1e-3)
    assert is_approx(db, g(c, "d_beta_exp"), 1e-3)


def test_gelu(O):
    c = "test_gelu.cpp::forward1"
    x = O.f32a(np.concatenate([g(c, "input[0]"), g(c, "input[1]")]))
    out = np.zeros_like(x)
    O.orc().orc_gelu_forward(out, x, x.size)
    for b in range(2):
        assert is_approx(out[12 * b:12 * b + 12], g(c, f"resexp[{b}]"), 1e-3)
    c = "test_gelu.cpp::backward1"
    x = O.f32a(np.concatenate([g(c, "input[0]"), g(c, "input[1]")]))
    d = np.zeros_like(x)
    O.orc().orc_gelu_backward(d, np.ones_like(x), x, x.size)
    for b in range(2):
        assert is_approx(d[12 * b:12 * b + 12], g(c, f"resexp[{b}]"), 1e-3)


def test_residual(O):
    c = "test_residual.cpp::forward1"
    a = O.f32a(np.concatenate([g(c, "input1[0]"), g(c, "input1[1]")]))
    b = O.f32a(np.concatenate([g(c, "input2[0]"), g(c, "input2[1]")]))
    out = np.zeros_like(a)
    O.orc().orc_residual_forward(out, a, b, a.size)
    for i in range(2):
        assert is_approx(out[12 * i:12 * i + 12], g(c, f"resexp[{i}]"), 1e-3)


def test_cross_entropy(O):
    c = "test_cross_entropy.cpp::forward1"
    tg = np.array(GOLD[c]["targets"], dtype=np.int32)
    probs = O.f32a(np.concatenate([g(c, "probs[0]", (7, 5)), g(c, "probs[1]", (7, 5))]))
    losses = np.zeros(14, np.float32)
    mean = O.orc().orc_cross_entropy(losses.ctypes.data, probs, tg, 14, 5)
    (e0, v0, t0), (e1, v1, t1) = GOLD[c]["EXPECT_NEAR"]
    assert abs(losses[:7].sum() / 7 - v0) < t0
    assert abs(losses[7:].sum() / 7 - v1) < t1
    assert abs(mean - (v0 + v1) / 2) < 1e-3


def test_encoder(O):
    c = "test_encoder.cpp::forward"
    tok = np.array(GOLD[c]["input"], dtype=np.int32)
    wte, wpe = g(c, "wte", (4, 3)), g(c, "wpe", (3, 3))
    out = np.zeros((2, 3, 3), np.float32)
    O.orc().orc_encoder_forward(out, tok, O.f32a(wte), O.f32a(wpe), 2, 3, 3)
    for b in range(2):
        np.testing.assert_array_equal(out[b], g(c, f"exp_res[{b}]", (3, 3)))
