"""Pins the oracle restatement to the reference's own compiled CPU code.

oracle/_ref/libref.so is the reference's gpt2/*.cpp built by
`make -C oracle ref` (needs the reference tree, so it is built in the
development container; skipped where it is absent). Inputs are seeded
normals from the oracle's generator; the metric is the hot path's max
relative error.
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref/libref.so not built here")


def mre(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


@pytest.mark.parametrize("B,T,C,OC", [(2, 64, 96, 160), (1, 37, 40, 24)])
def test_matmul_vs_ref(B, T, C, OC):
    x = O.normal((B * T, C), 11)
    W = O.normal((OC, C), 12)
    b = O.normal((OC,), 13)
    dout = O.normal((B * T, OC), 14)
    y_o = np.zeros((B * T, OC), np.float32)
    y_r = np.zeros_like(y_o)
    O.orc().orc_matmul_forward(y_o, x, W, b.ctypes.data, B * T, C, OC)
    O.ref().ref_matmul_forward(y_r, x, W, b.ctypes.data, B, T, C, OC)
    assert mre(y_o, y_r) < 1e-5
    di_o, dw_o, db_o = np.zeros((B * T, C), np.float32), np.zeros((OC, C), np.float32), np.zeros(OC, np.float32)
    di_r, dw_r, db_r = np.zeros_like(di_o), np.zeros_like(dw_o), np.zeros_like(db_o)
    O.orc().orc_matmul_backward(di_o, dw_o, db_o.ctypes.data, dout, x, W, B * T, C, OC)
    O.ref().ref_matmul_backward(di_r, dw_r, db_r, dout, x, W, B, T, C, OC)
    assert mre(di_o, di_r) < 1e-5 and mre(dw_o, dw_r) < 1e-5 and mre(db_o, db_r) < 1e-5


@pytest.mark.parametrize("B,T,C,NH", [(2, 64, 128, 2), (1, 33, 64, 1)])
def test_attention_vs_ref(B, T, C, NH):
    qkv = O.normal((B, T, 3 * C), 21)
    dout = O.normal((B, T, C), 22)
    out_o = np.zeros((B, T, C), np.float32)
    att_o = np.zeros((B, NH, T, T), np.float32)
    out_r = np.zeros_like(out_o)
    att_r = np.zeros_like(att_o)
    O.orc().orc_attention_forward(out_o, att_o, None, qkv, B, T, C, NH)
    O.ref().ref_attention_forward(out_r, att_r.ctypes.data, qkv, B, T, C, NH)
    assert mre(out_o, out_r) < 1e-5 and mre(att_o, att_r) < 1e-5
    d_o = np.zeros((B, T, 3 * C), np.float32)
    d_r = np.zeros_like(d_o)
    O.orc().orc_attention_backward(d_o, dout, qkv, att_o, B, T, C, NH)
    O.ref().ref_attention_backward(d_r, dout, qkv, B, T, C, NH)
    assert mre(d_o, d_r) < 1e-4


def test_layernorm_gelu_vs_ref():
    B, T, C = 2, 48, 160
    x = O.normal((B * T, C), 31, std=3.0)
    gm = O.normal((C,), 32)
    bt = O.normal((C,), 33)
    dy = O.normal((B * T, C), 34)
    y_o, y_r = np.zeros_like(x), np.zeros_like(x)
    m_o, r_o = np.zeros(B * T, np.float32), np.zeros(B * T, np.float32)
    m_r, r_r = np.zeros_like(m_o), np.zeros_like(r_o)
    O.orc().orc_layernorm_forward(y_o, m_o.ctypes.data, r_o.ctypes.data, x, gm, bt, B * T, C)
    O.ref().ref_layernorm_forward(y_r, m_r, r_r, x, gm, bt, B, T, C)
    assert mre(y_o, y_r) < 1e-5
    dx_o, dg_o, db_o = np.zeros_like(x), np.zeros(C, np.float32), np.zeros(C, np.float32)
    dx_r, dg_r, db_r = np.zeros_like(x), np.zeros(C, np.float32), np.zeros(C, np.float32)
    O.orc().orc_layernorm_backward(dx_o, dg_o, db_o, dy, x, gm, m_o, r_o, B * T, C)
    O.ref().ref_layernorm_backward(dx_r, dg_r, db_r, dy, x, gm, bt, B, T, C)
    assert mre(dx_o, dx_r) < 1e-4 and mre(dg_o, dg_r) < 1e-5 and mre(db_o, db_r) < 1e-5
    g_o, g_r = np.zeros_like(x), np.zeros_like(x)
    O.orc().orc_gelu_forward(g_o, x, x.size)
    O.ref().ref_gelu_forward(g_r, x, B, T, C)
    assert mre(g_o, g_r) < 1e-5
    O.orc().orc_gelu_backward(g_o, dy, x, x.size)
    O.ref().ref_gelu_backward(g_r, dy, x, B, T, C)
    assert mre(g_o, g_r) < 1e-5


def test_gpt2_small_training_vs_ref(tmp_path):
    """A 2-layer GPT-2 (C=128, V=1000) trained 5 steps by both: losses within 1e-4 relative."""
    cfg = O.config(max_seq_len=64, vocab_size=1000, padded_vocab_size=1024, num_layers=2, num_heads=4, channels=128)
    B, T = 2, 32
    params = O.init_params(cfg, 1337)
    ckpt = str(tmp_path / "small.bin")
    O.write_checkpoint(ckpt, cfg, params)
    toks = O.tokens(B * T + 1, cfg.vocab_size, 1337)
    inp, tgt = toks[:-1].copy(), toks[1:].copy()
    steps = 5
    ref_losses = np.zeros(steps, np.float32)
    ms = np.zeros(steps, np.float64)
    O.ref().ref_gpt2_train(ckpt.encode(), B, T, inp, tgt, steps, 3e-4, ref_losses, ms)
    m = O.Model(cfg, params, B, T)
    for s in range(steps):
        loss = m.forward(inp, tgt)
        m.zero_grad()
        m.backward()
        m.update(3e-4, t=s + 1)
        assert abs(loss - ref_losses[s]) / ref_losses[s] < 1e-4, (s, loss, ref_losses[s])
