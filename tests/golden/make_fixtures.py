"""Generates the committed golden fixtures from the reference's compiled CPU code.

    make -C oracle ref && python tests/golden/make_fixtures.py

gpt2_124m_b4t64_losses.json — configuration 0 of the benchmark spec: GPT-2
124M (L=12, NH=12, C=768, V=50257, Vp=50304, maxT=1024) initialised from
seed 1337 by orc_gpt2_init_params (weights N(0, 0.02), projection weights
scaled by 1/sqrt(2L), biases 0, LayerNorm 1/0, padded vocab rows 0), written
as an llm.c v3 checkpoint and loaded by the reference's own GPT2 loader.
Tokens: B*T+1 = 257 uniform int32 in [0, 50257) from seed 1337 (stream 1);
inputs = tokens[0:256], targets = tokens[1:257]; the same batch every step.
20 steps of Forward / ZeroGrad / Backward / Update(lr=3e-4, 0.9, 0.999, 1e-8,
wd=0, t=step+1), the loop of train.cpp:123-146. Records the reference's mean
loss per step.
"""
from __future__ import annotations

import json
import os
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle as O  # noqa: E402

SEED, B, T, STEPS, LR = 1337, 4, 64, 20, 3e-4


def config0_batch(cfg):
    toks = O.tokens(B * T + 1, cfg.vocab_size, SEED)
    return toks[:-1].copy(), toks[1:].copy()


def main() -> None:
    cfg = O.config()
    params = O.init_params(cfg, SEED)
    inp, tgt = config0_batch(cfg)
    with tempfile.TemporaryDirectory() as d:
        ckpt = os.path.join(d, "gpt2_124m_seed1337.bin")
        O.write_checkpoint(ckpt, cfg, params)
        losses = np.zeros(STEPS, np.float32)
        ms = np.zeros(STEPS, np.float64)
        t0 = time.time()
        O.ref().ref_gpt2_train(ckpt.encode(), B, T, inp, tgt, STEPS, LR, losses, ms)
        wall = time.time() - t0
    out = {
        "description": "reference CPU (llm.cpp gpt2/*.cpp, -O3 -ffast-math -fopenmp) loss per step, config 0",
        "seed": SEED, "B": B, "T": T, "steps": STEPS, "lr": LR,
        "param_checksum": float(np.float64(params).sum()),
        "tokens_head": inp[:8].tolist(),
        "losses": [float(x) for x in losses],
        "step_ms": [float(x) for x in ms],
        "cores": os.cpu_count(),
        "wall_s": wall,
    }
    with open(os.path.join(HERE, "gpt2_124m_b4t64_losses.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(json.dumps({k: out[k] for k in ("losses", "wall_s")}, indent=1))


if __name__ == "__main__":
    main()
