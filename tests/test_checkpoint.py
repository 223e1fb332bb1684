"""Model files (llm.c v3, the format the reference's GPT2 constructors read,
gpt2/cuda/gpt2cuda.cu:33-166 and gpt2/gpt2.cpp:112-230) and training-state
files: header parsing and validation on CPU; load / save / resume through the
model on the GPU.

The model files written here are the oracle's (oracle.write_checkpoint, the
field order of gpt2/gpt2.cpp:118-135); the reference harness trains from a
file this library saved to show the reference reads it."""
import ctypes
import os

import numpy as np
import pytest

import oracle as O

SMALL = dict(max_seq_len=128, vocab_size=1000, padded_vocab_size=1024, num_layers=2, num_heads=2, channels=128)


def _cfg_tuple(c):
    return (c.max_seq_len, c.vocab_size, c.padded_vocab_size, c.num_layers, c.num_heads, c.channels)


def _model(llmk, cfg, B, T, math):
    return llmk.GPT2(B, T, max_seq_len=cfg.max_seq_len, vocab_size=cfg.vocab_size,
                     padded_vocab_size=cfg.padded_vocab_size, num_layers=cfg.num_layers, num_heads=cfg.num_heads,
                     channels=cfg.channels, math=math)


# ------------------------------------------------------------------- CPU
def test_checkpoint_config_reads_header(tmp_path, llmk_lib):
    import llmk
    cfg = O.config(**SMALL)
    p = str(tmp_path / "m.bin")
    O.write_checkpoint(p, cfg, O.init_params(cfg, 1))
    c = llmk.checkpoint_config(p)
    assert _cfg_tuple(c) == _cfg_tuple(cfg)
    n = llmk.lib().llmk_gpt2_num_parameters(ctypes.byref(c))
    assert os.path.getsize(p) == 1024 + 4 * n


def test_checkpoint_header_errors(tmp_path, llmk_lib):
    import llmk
    cfg = O.config(**SMALL)
    params = O.init_params(cfg, 1)
    good = str(tmp_path / "good.bin")
    O.write_checkpoint(good, cfg, params)
    raw = bytearray(open(good, "rb").read())

    def variant(name, mutate):
        b = bytearray(raw)
        mutate(b)
        q = str(tmp_path / name)
        open(q, "wb").write(bytes(b))
        return q

    bad_magic = variant("magic.bin", lambda b: b.__setitem__(slice(0, 4), np.int32(20240520).tobytes()))
    with pytest.raises(llmk.LlmkError, match="bad magic"):
        llmk.checkpoint_config(bad_magic)
    bad_version = variant("version.bin", lambda b: b.__setitem__(slice(4, 8), np.int32(2).tobytes()))
    with pytest.raises(llmk.LlmkError, match="bad version"):
        llmk.checkpoint_config(bad_version)
    truncated = variant("short.bin", lambda b: b.__delitem__(slice(len(b) - 4, len(b))))
    with pytest.raises(llmk.LlmkError, match="file size"):
        llmk.checkpoint_config(truncated)
    bad_cfg = variant("cfg.bin", lambda b: b.__setitem__(slice(20, 24), np.int32(3).tobytes()))  # NH = 3
    with pytest.raises(llmk.LlmkError, match="bad configuration"):
        llmk.checkpoint_config(bad_cfg)
    with pytest.raises(llmk.LlmkError, match="cannot open"):
        llmk.checkpoint_config(str(tmp_path / "missing.bin"))
    # a training-state file is not a model file
    st = variant("state.bin", lambda b: b.__setitem__(slice(0, 4), np.int32(20241202).tobytes()))
    with pytest.raises(llmk.LlmkError, match="bad magic"):
        llmk.checkpoint_config(st)


# ------------------------------------------------------------------- GPU
@pytest.mark.gpu
def test_load_and_save_roundtrip(cuda_dev, tmp_path):
    import llmk
    cfg = O.config(**SMALL)
    params = O.init_params(cfg, 3)
    src = str(tmp_path / "in.bin")
    O.write_checkpoint(src, cfg, params)
    m = llmk.GPT2.from_checkpoint(src, 2, 64)
    assert _cfg_tuple(m.cfg) == _cfg_tuple(cfg)
    assert np.array_equal(m.read_parameters(), params)
    out = str(tmp_path / "out.bin")
    m.save_checkpoint(out)
    assert open(out, "rb").read() == open(src, "rb").read()  # byte-identical to the oracle's writer
    assert not os.path.exists(out + ".tmp")
    # a file of another configuration is refused, the model is left as it was
    other = O.config(**dict(SMALL, num_layers=3))
    q = str(tmp_path / "other.bin")
    O.write_checkpoint(q, other, O.init_params(other, 4))
    with pytest.raises(llmk.LlmkError, match="configuration differs"):
        m.load_checkpoint(q)
    assert np.array_equal(m.read_parameters(), params)
    m.close()


@pytest.mark.gpu
@pytest.mark.skipif(not O.ref_available(), reason="reference library not built")
def test_reference_trains_from_saved_checkpoint(cuda_dev, tmp_path):
    """After a few steps here, the saved model file is read by the reference's
    own GPT2 constructor: its first loss equals the oracle's loss on the
    parameters this library holds."""
    import llmk
    cfg = O.config(**SMALL)
    B, T = 2, 64
    params = O.init_params(cfg, 5)
    toks = O.tokens(B * T + 1, cfg.vocab_size, 5)
    inp, tgt = toks[:-1].copy(), toks[1:].copy()
    m = _model(llmk, cfg, B, T, llmk.MATH_TF32)
    m.load_parameters(params)
    for s in range(3):
        m.train_step(inp, tgt, 1e-3, t=s + 1)
    p = str(tmp_path / "trained.bin")
    m.save_checkpoint(p)
    trained = m.read_parameters()
    m.close()
    losses = np.zeros(1, np.float32)
    ms = np.zeros(1, np.float64)
    assert O.ref().ref_gpt2_train(p.encode(), B, T, inp, tgt, 1, 0.0, losses, ms) == 0
    oracle_loss = O.Model(cfg, trained, B, T).forward(inp, tgt)
    assert abs(losses[0] - oracle_loss) / oracle_loss < 1e-4, (losses[0], oracle_loss)


@pytest.mark.gpu
@pytest.mark.parametrize("mathname", ["bf16", "tf32"])
def test_state_resume_continues_training(cuda_dev, tmp_path, mathname):
    """Train 6 steps, saving the state after 3; load it into a fresh model and
    train the last 3 again: the resumed losses follow the first run. (Not
    bit-exact: split-K partial sums and the dQ accumulation add in
    scheduling order.)"""
    import llmk
    math = llmk.MATH_TF32 if mathname == "tf32" else llmk.MATH_BF16
    cfg = O.config(**SMALL)
    B, T = 2, 64
    params = O.init_params(cfg, 9)
    toks = O.tokens(B * T * 6 + 1, cfg.vocab_size, 9)
    batches = [(toks[i * B * T:(i + 1) * B * T].copy(), toks[i * B * T + 1:(i + 1) * B * T + 1].copy())
               for i in range(6)]
    st = str(tmp_path / "state.bin")
    a = _model(llmk, cfg, B, T, math)
    a.load_parameters(params)
    straight = []
    for s, (i, t) in enumerate(batches):
        if s == 3:
            a.save_state(st, step=3, loader_position=(2, 7), world=1)
            m_a, v_a = a.read_optimizer_state()
            p_a = a.read_parameters()
        straight.append(a.train_step(i, t, 1e-3, t=s + 1, wd=0.1))
    a.close()
    c = _model(llmk, cfg, B, T, math)
    info = c.load_state(st)
    assert info == {"step": 3, "world": 1, "loader_position": (2, 7)}
    m_c, v_c = c.read_optimizer_state()
    assert np.array_equal(m_c, m_a) and np.array_equal(v_c, v_a) and np.array_equal(c.read_parameters(), p_a)
    assert np.any(m_c != 0) and np.all(v_c >= 0)
    resumed = [c.train_step(i, t, 1e-3, t=info["step"] + s + 1, wd=0.1) for s, (i, t) in enumerate(batches[3:])]
    rel = [abs(x - y) / y for x, y in zip(resumed, straight[3:])]
    assert rel[0] < 1e-5 and max(rel) < 1e-4, (rel, resumed, straight[3:])
    # a fresh model that skipped the state (zero moments, t = 1) takes another path
    d = _model(llmk, cfg, B, T, math)
    d.load_parameters(p_a)
    other = [d.train_step(i, t, 1e-3, t=s + 1, wd=0.1) for s, (i, t) in enumerate(batches[3:])]
    assert abs(other[-1] - straight[-1]) / straight[-1] > 10 * max(rel)
    d.close()
    # a model file is not a state file
    with pytest.raises(llmk.LlmkError, match="bad magic"):
        c.load_state(_write_model(tmp_path, cfg, params))
    c.close()


def _write_model(tmp_path, cfg, params):
    p = str(tmp_path / "model.bin")
    O.write_checkpoint(p, cfg, params)
    return p
