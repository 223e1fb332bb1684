"""End-to-end GPT-2 training on the GPU vs the reference's fp32 CPU path.

test_config0_loss_trajectory: configuration 0 of the benchmark spec (GPT-2
124M, B=4, T=64, seed 1337, AdamW lr 3e-4, 20 steps on one fixed batch).
The expected losses are the reference's own (llm.cpp gpt2/*.cpp compiled and
run by tests/golden/make_fixtures.py). In TF32 mode (fp32 activations, TF32
GEMMs: the reference GPU path's precision) the bar is |L_gpu - L_ref| / L_ref
<= 0.5% at every step, for both modes: TF32 (fp32 activations, TF32 GEMMs:
the reference GPU path's precision) and bf16 (bf16 GEMM operands and
activations, fp32 master weights: what the benchmark runs).

The bf16 run has little margin (about 0.5% at its worst step, measured on a
B200). That is bf16 arithmetic, not a kernel fault: the run overfits one batch
from loss 11 to 2 in 20 steps, so any rounding perturbation grows along the
trajectory. tests/golden/bf16_drift.py replays the same 20 steps in fp32
torch on the CPU with bf16 rounding at the points the device rounds; its
committed result (tests/golden/gpt2_124m_b4t64_bf16_drift.json) shows 0.3-0.6%
worst-step drift from rounding the weights alone, the activations alone, or
everything, against 0.003% for the unrounded fp32 replay.
"""
import json
import os

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _model(llmk, cfg, B, T, math):
    return llmk.GPT2(B, T, max_seq_len=cfg.max_seq_len, vocab_size=cfg.vocab_size,
                     padded_vocab_size=cfg.padded_vocab_size, num_layers=cfg.num_layers, num_heads=cfg.num_heads,
                     channels=cfg.channels, math=math)


@pytest.mark.parametrize("mathname,bar", [("tf32", 5e-3), ("bf16", 5e-3)])
def test_config0_loss_trajectory(cuda_dev, mathname, bar):
    import llmk
    math = llmk.MATH_TF32 if mathname == "tf32" else llmk.MATH_BF16
    fx = json.load(open(os.path.join(HERE, "golden", "gpt2_124m_b4t64_losses.json")))
    cfg = O.config()
    B, T, steps = fx["B"], fx["T"], fx["steps"]
    params = O.init_params(cfg, fx["seed"])
    assert abs(float(np.float64(params).sum()) - fx["param_checksum"]) < 1e-6 * max(1.0, abs(fx["param_checksum"]))
    toks = O.tokens(B * T + 1, cfg.vocab_size, fx["seed"])
    assert toks[:8].tolist() == fx["tokens_head"]
    inp, tgt = toks[:-1], toks[1:]
    m = _model(llmk, cfg, B, T, math)
    m.load_parameters(params)
    losses = [m.train_step(inp, tgt, fx["lr"], t=s + 1) for s in range(steps)]
    ref = fx["losses"]
    rel = [abs(a - b) / b for a, b in zip(losses, ref)]
    print(mathname, "gpu", [round(x, 4) for x in losses])
    print(mathname, "ref", [round(x, 4) for x in ref])
    print(mathname, "rel", [f"{x:.2e}" for x in rel])
    assert max(rel) <= bar, rel
    assert llmk.device_status() == 0
    m.close()


@pytest.mark.parametrize("mathname,tol", [("tf32", 1e-2), ("bf16", 5e-2)])
def test_small_model_gradients_vs_oracle(cuda_dev, mathname, tol):
    """One forward/backward of a 2-layer model: loss and every gradient tensor vs the oracle
    (norm-wise relative error, the reference tests' isApprox metric)."""
    import llmk
    math = llmk.MATH_TF32 if mathname == "tf32" else llmk.MATH_BF16
    cfg = O.config(max_seq_len=128, vocab_size=1000, padded_vocab_size=1024, num_layers=2, num_heads=2, channels=128)
    B, T = 2, 128
    params = O.init_params(cfg, 7)
    toks = O.tokens(B * T + 1, cfg.vocab_size, 7)
    inp, tgt = toks[:-1].copy(), toks[1:].copy()
    ref = O.Model(cfg, params, B, T)
    loss_ref = ref.forward(inp, tgt)
    ref.zero_grad()
    ref.backward()
    g_ref = ref.grads()
    m = _model(llmk, cfg, B, T, math)
    m.load_parameters(params)
    # lr = 0: the step leaves the parameters unchanged and exposes the gradients
    loss = m.train_step(inp, tgt, 0.0, t=1)
    g = m.read_gradients()
    assert abs(loss - loss_ref) / loss_ref < (1e-3 if mathname == "tf32" else 1e-2), (loss, loss_ref)
    sizes = O.param_sizes(cfg)
    names = ["wte", "wpe", "ln1w", "ln1b", "qkvw", "qkvb", "attprojw", "attprojb", "ln2w", "ln2b", "fcw", "fcb",
             "fcprojw", "fcprojb", "lnfw", "lnfb"]
    off = 0
    for name, n in zip(names, sizes):
        a, b = g[off:off + n].astype(np.float64), g_ref[off:off + n].astype(np.float64)
        off += n
        nrm = np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)
        assert nrm < tol, f"{name}: norm-rel err {nrm:.3e}"
    assert np.array_equal(m.read_parameters(), params)
    m.close()


@pytest.mark.parametrize("mathname", ["bf16", "tf32"])
def test_repeated_steps_agree(cuda_dev, mathname):
    """The same step (lr = 0) repeated five times gives the same gradients: a
    race between kernels, streams or CTAs shows up as run-to-run spread (the
    only unordered sum is the attention dQ reduction, ~1e-7 relative)."""
    import llmk
    math = llmk.MATH_TF32 if mathname == "tf32" else llmk.MATH_BF16
    cfg = O.config(max_seq_len=128, vocab_size=1000, padded_vocab_size=1024, num_layers=2, num_heads=2, channels=128)
    B, T = 2, 128
    params = O.init_params(cfg, 11)
    toks = O.tokens(B * T + 1, cfg.vocab_size, 11)
    m = _model(llmk, cfg, B, T, math)
    m.load_parameters(params)
    first = None
    for _ in range(5):
        m.train_step(toks[:-1], toks[1:], 0.0, t=1)
        g = m.read_gradients().astype(np.float64)
        if first is None:
            first = g
        else:
            err = np.abs(g - first).max() / np.abs(first).max()
            assert err < 1e-5, err
    m.close()


def test_step_timing_report(cuda_dev):
    """Per-kernel-class step timing: every GEMM of the step is counted once per
    step with its 2*M*N*K FLOPs, and timing does not change the step's result."""
    import llmk
    cfg = O.config(max_seq_len=128, vocab_size=1000, padded_vocab_size=1024, num_layers=2, num_heads=2, channels=128)
    B, T = 2, 128
    params = O.init_params(cfg, 12)
    toks = O.tokens(B * T + 1, cfg.vocab_size, 12)
    m = _model(llmk, cfg, B, T, llmk.MATH_BF16)
    m.load_parameters(params)
    m.train_step(toks[:-1], toks[1:], 0.0, t=1)
    g0 = m.read_gradients()
    m.set_timing(True)
    for _ in range(2):
        m.train_step(toks[:-1], toks[1:], 0.0, t=1)
    rep = m.timing_report()
    m.set_timing(False)
    assert np.array_equal(m.read_gradients(), g0)
    L, C, Vp, BT = cfg.num_layers, cfg.channels, cfg.padded_vocab_size, B * T
    per_layer = 2 * BT * C * (3 * C + C + 4 * C + 4 * C)  # forward MACs x 2 of qkv, attproj, fc, fcproj
    flop = 3 * (L * per_layer + 2 * BT * Vp * C)  # forward, dinp, dweight
    for name, calls in (("gemm_fwd", 4 * L), ("gemm_dinp", 4 * L), ("gemm_dweight", 4 * L), ("gemm_lm_head", 3)):
        assert rep[name]["calls"] == 2 * calls and rep[name]["unit"] == "flop", name
        assert rep[name]["ms"] > 0 and rep[name]["launches"] >= rep[name]["calls"], name
    gemm_work = sum(rep[n]["work"] for n in ("gemm_fwd", "gemm_dinp", "gemm_dweight", "gemm_lm_head"))
    assert abs(gemm_work - 2 * flop) <= 1e-9 * flop
    assert abs(rep["gemm_lm_head"]["work"] - 2 * 3 * 2 * BT * Vp * C) <= 1e-9 * flop
    for name in ("attention_fwd", "attention_bwd", "layernorm_fwd", "layernorm_bwd", "adamw", "softmax_xent"):
        assert rep[name]["calls"] > 0 and rep[name]["ms"] > 0, name
    assert rep["attention_fwd"]["calls"] == 2 * L
    m.set_timing(True)
    assert m.timing_report()["gemm_fwd"]["calls"] == 0
    m.close()


@pytest.mark.parametrize("mathname", ["bf16", "tf32"])
def test_graph_steps_match_eager(cuda_dev, mathname):
    """CUDA-graph mode: captured steps (the AdamW step count and learning rate
    changing per replay) give the eager steps' losses and parameters."""
    import llmk
    math = llmk.MATH_TF32 if mathname == "tf32" else llmk.MATH_BF16
    cfg = O.config(max_seq_len=128, vocab_size=1000, padded_vocab_size=1024, num_layers=2, num_heads=2, channels=128)
    B, T = 2, 128
    params = O.init_params(cfg, 13)
    toks = O.tokens(4 * B * T + 1, cfg.vocab_size, 13)
    runs = []
    for graph in (False, True):
        m = _model(llmk, cfg, B, T, math)
        m.load_parameters(params)
        m.use_graph(graph)
        losses = []
        for step in range(4):
            c = toks[step * B * T:(step + 1) * B * T + 1]
            losses.append(m.train_step(c[:-1], c[1:], 1e-3 * (step + 1), t=step + 1))
        runs.append((np.array(losses), m.read_parameters()))
        m.close()
    (l0, p0), (l1, p1) = runs
    assert np.allclose(l0, l1, rtol=1e-5, atol=0), (l0, l1)
    assert np.abs(p1 - p0).max() / np.abs(p0).max() < 1e-4
    assert llmk.device_status() == 0


_CONFIG3_REF = {}


def _config3_oracle():
    """The oracle's loss and gradients of one GPT-2 124M step at T = 1024
    (configuration 3's sequence length and model; B = 1, seed 31)."""
    if not _CONFIG3_REF:
        cfg = O.config()
        B, T = 1, 1024
        params = O.init_params(cfg, 31)
        toks = O.tokens(B * T + 1, cfg.vocab_size, 31)
        ref = O.Model(cfg, params, B, T)
        loss = ref.forward(toks[:-1], toks[1:])
        ref.zero_grad()
        ref.backward()
        _CONFIG3_REF.update(cfg=cfg, B=B, T=T, params=params, toks=toks, loss=loss, grads=ref.grads())
        del ref
    return _CONFIG3_REF


@pytest.mark.parametrize("mathname,ltol,gtol", [("bf16", 1e-2, 5e-2), ("tf32", 1e-3, 1e-2)])
def test_config3_step_vs_oracle(cuda_dev, mathname, ltol, gtol):
    """Configuration 3's model at its full sequence length: one GPT-2 124M
    training step (B = 1, T = 1024) through the native trainer against the
    oracle — loss and every parameter gradient (norm-wise relative error, the
    reference tests' isApprox metric; the max relative error is printed)."""
    import llmk
    math = llmk.MATH_TF32 if mathname == "tf32" else llmk.MATH_BF16
    r = _config3_oracle()
    cfg, B, T = r["cfg"], r["B"], r["T"]
    m = _model(llmk, cfg, B, T, math)
    m.load_parameters(r["params"])
    loss = m.train_step(r["toks"][:-1], r["toks"][1:], 0.0, t=1)
    g = m.read_gradients()
    m.close()
    assert abs(loss - r["loss"]) / r["loss"] < ltol, (loss, r["loss"])
    names = ["wte", "wpe", "ln1w", "ln1b", "qkvw", "qkvb", "attprojw", "attprojb", "ln2w", "ln2b", "fcw", "fcb",
             "fcprojw", "fcprojb", "lnfw", "lnfb"]
    off = 0
    report = {}
    for name, n in zip(names, O.param_sizes(cfg)):
        a, b = g[off:off + n].astype(np.float64), r["grads"][off:off + n].astype(np.float64)
        off += n
        nrm = np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)
        mx = np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)
        report[name] = (nrm, mx)
    print(mathname, f"loss {loss:.6f} oracle {r['loss']:.6f}",
          {k: f"{v[0]:.1e}/{v[1]:.1e}" for k, v in report.items()})
    for name, (nrm, mx) in report.items():
        assert nrm < gtol, f"{name}: norm-rel err {nrm:.3e}"
    assert llmk.device_status() == 0


@pytest.mark.parametrize("mathname,tol", [("bf16", 5e-2), ("tf32", 1e-2)])
def test_774m_shape_gradients_vs_oracle(cuda_dev, mathname, tol):
    """Configuration 4's layer shape (C = 1280, NH = 20, head size 64: K = 1280
    GEMMs, 20-head attention, 1280-wide LayerNorms) in a 2-layer model, one
    step against the oracle: loss and every gradient tensor."""
    import llmk
    math = llmk.MATH_TF32 if mathname == "tf32" else llmk.MATH_BF16
    cfg = O.config(max_seq_len=256, vocab_size=1000, padded_vocab_size=1024, num_layers=2, num_heads=20,
                   channels=1280)
    B, T = 2, 256
    params = O.init_params(cfg, 41)
    toks = O.tokens(B * T + 1, cfg.vocab_size, 41)
    ref = O.Model(cfg, params, B, T)
    loss_ref = ref.forward(toks[:-1], toks[1:])
    ref.zero_grad()
    ref.backward()
    g_ref = ref.grads()
    m = _model(llmk, cfg, B, T, math)
    m.load_parameters(params)
    loss = m.train_step(toks[:-1], toks[1:], 0.0, t=1)
    g = m.read_gradients()
    m.close()
    assert abs(loss - loss_ref) / loss_ref < (1e-3 if mathname == "tf32" else 1e-2), (loss, loss_ref)
    names = ["wte", "wpe", "ln1w", "ln1b", "qkvw", "qkvb", "attprojw", "attprojb", "ln2w", "ln2b", "fcw", "fcb",
             "fcprojw", "fcprojb", "lnfw", "lnfb"]
    off = 0
    for name, n in zip(names, O.param_sizes(cfg)):
        a, b = g[off:off + n].astype(np.float64), g_ref[off:off + n].astype(np.float64)
        off += n
        if name == "wpe":  # rows beyond T have zero gradient in both
            a, b = a[:T * cfg.channels], b[:T * cfg.channels]
        nrm = np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)
        assert nrm < tol, f"{name}: norm-rel err {nrm:.3e}"
    assert llmk.device_status() == 0
