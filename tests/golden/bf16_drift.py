"""bf16 comparator for the configuration-0 loss trajectory (TEST INFRASTRUCTURE).

    python tests/golden/bf16_drift.py [variant ...]

Replays configuration 0 of the benchmark spec (GPT-2 124M, B=4, T=64, seed
1337, AdamW lr 3e-4, 20 steps on one fixed batch; initial parameters and
tokens from the oracle's seeded generator, so the same bytes the reference
run in gpt2_124m_b4t64_losses.json consumed) as an fp32 torch model on the
CPU, with bf16 rounding (round to nearest even) inserted where the device's
bf16 mode rounds:

  weights      the bf16 copy of every GEMM weight (fp32 master kept for AdamW)
  activations  every GEMM / attention operand stored in bf16 (LayerNorm
               outputs, q/k/v, attention output, GELU output, pre-activation)
  gradients    every activation gradient stored in bf16 before a GEMM reads it
  logits       the bf16 logits buffer
  attention_p  softmax probabilities and dS rounded for the attention MMAs

and writes the per-step relative loss error against the reference's own
losses for each variant to gpt2_124m_b4t64_bf16_drift.json. The unrounded
replay ("fp32") pins the replay itself to the reference. It separates
bf16 arithmetic drift from kernel faults: a device run whose worst-step error
is of the size the rounded replays show is drifting, not wrong.
"""
from __future__ import annotations

import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (ROOT, os.path.join(ROOT, "llm.cpp_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

import oracle as O  # noqa: E402

VARIANTS = {
    "fp32": {},
    "weights": {"w": 1},
    "activations": {"act": 1},
    "gradients": {"grad": 1},
    "logits": {"logits": 1},
    "attention_p": {"attp": 1},
    "all": {"w": 1, "act": 1, "grad": 1, "logits": 1, "attp": 1},
}


class _RoundValue(torch.autograd.Function):
    """bf16-rounds the value; the gradient passes unchanged."""

    @staticmethod
    def forward(ctx, x):
        return x.bfloat16().float()

    @staticmethod
    def backward(ctx, g):
        return g


class _RoundGrad(torch.autograd.Function):
    """Leaves the value; bf16-rounds the gradient flowing back through it."""

    @staticmethod
    def forward(ctx, x):
        return x.clone()

    @staticmethod
    def backward(ctx, g):
        return g.bfloat16().float()


def replay(flags: dict, fx: dict) -> list[float]:
    cfg = O.config()
    B, T = fx["B"], fx["T"]
    L, C, NH, Vp, V, maxT = (cfg.num_layers, cfg.channels, cfg.num_heads, cfg.padded_vocab_size, cfg.vocab_size,
                             cfg.max_seq_len)
    params = O.init_params(cfg, fx["seed"])
    toks = O.tokens(B * T + 1, V, fx["seed"])
    inp = torch.from_numpy(toks[:-1].astype(np.int64)).view(B, T)
    tgt = torch.from_numpy(toks[1:].astype(np.int64)).view(B, T)
    sizes = O.param_sizes(cfg)
    p = torch.from_numpy(params.copy())
    m = torch.zeros_like(p)
    v = torch.zeros_like(p)
    ident = lambda x: x  # noqa: E731
    rv = lambda x: _RoundValue.apply(x)  # noqa: E731
    rg = lambda x: _RoundGrad.apply(x)  # noqa: E731
    rw = rv if flags.get("w") else ident
    ra = rv if flags.get("act") else ident
    rgr = rg if flags.get("grad") else ident
    rl = rv if flags.get("logits") else ident
    rp = rv if flags.get("attp") else ident
    rs = rg if flags.get("attp") else ident
    hd = C // NH
    mask = torch.ones(T, T, dtype=torch.bool).tril()
    losses = []
    for step in range(fx["steps"]):
        pp = p.clone().requires_grad_(True)
        parts = torch.split(pp, sizes)
        wte, wpe = parts[0].view(Vp, C), parts[1].view(maxT, C)
        ln1w, ln1b = parts[2].view(L, C), parts[3].view(L, C)
        qkvw, qkvb = parts[4].view(L, 3 * C, C), parts[5].view(L, 3 * C)
        apw, apb = parts[6].view(L, C, C), parts[7].view(L, C)
        ln2w, ln2b = parts[8].view(L, C), parts[9].view(L, C)
        fcw, fcb = parts[10].view(L, 4 * C, C), parts[11].view(L, 4 * C)
        fpw, fpb = parts[12].view(L, C, 4 * C), parts[13].view(L, C)
        lnfw, lnfb = parts[14], parts[15]

        def ln(x, w, b):  # two-pass variance, eps 1e-5 (gpt2/layernorm.cpp:16-23)
            mu = x.mean(-1, keepdim=True)
            var = ((x - mu) ** 2).mean(-1, keepdim=True)
            return (x - mu) * torch.rsqrt(var + 1e-5) * w + b

        def lin(x, W, b=None):
            y = ra(x) @ rw(W).t()
            return y + b if b is not None else y

        x = wte[inp] + wpe[:T]
        for li in range(L):
            qkv = ra(rgr(lin(ln(x, ln1w[li], ln1b[li]), qkvw[li], qkvb[li])))
            q, k, vv = (t.view(B, T, NH, hd).transpose(1, 2) for t in qkv.split(C, -1))
            s = rs((q @ k.transpose(-1, -2)) / hd ** 0.5).masked_fill(~mask, float("-inf"))
            o = (rp(torch.softmax(s, -1)) @ vv).transpose(1, 2).reshape(B, T, C)
            x = x + rgr(lin(ra(rgr(o)), apw[li], apb[li]))
            pre = ra(lin(ln(x, ln2w[li], ln2b[li]), fcw[li], fcb[li]))
            g = 0.5 * pre * (1 + torch.tanh((2 / np.pi) ** 0.5 * (pre + 0.044715 * pre ** 3)))
            x = x + rgr(lin(ra(rgr(g)), fpw[li], fpb[li]))
        logits = rl(rgr(lin(ln(x, lnfw, lnfb), wte)))
        loss = torch.nn.functional.cross_entropy(logits[..., :V].reshape(-1, V), tgt.reshape(-1))
        loss.backward()
        losses.append(loss.item())
        gr = pp.grad.detach()
        t = step + 1
        b1, b2, eps = 0.9, 0.999, 1e-8
        m = b1 * m + (1 - b1) * gr
        v = b2 * v + (1 - b2) * gr * gr
        p = p - fx["lr"] * ((m / (1 - b1 ** t)) / ((v / (1 - b2 ** t)).sqrt() + eps))
    return losses


def main(names: list[str]) -> None:
    torch.set_num_threads(os.cpu_count() or 1)
    fx = json.load(open(os.path.join(HERE, "gpt2_124m_b4t64_losses.json")))
    ref = fx["losses"]
    out_path = os.path.join(HERE, "gpt2_124m_b4t64_bf16_drift.json")
    out = json.load(open(out_path)) if os.path.exists(out_path) else {
        "description": "configuration-0 loss trajectory replayed in fp32 torch on the CPU with bf16 rounding at "
                       "the device's rounding points; rel = |L - L_ref| / L_ref per step against the reference's "
                       "losses (gpt2_124m_b4t64_losses.json)", "variants": {}}
    for name in names:
        t0 = time.time()
        losses = replay(VARIANTS[name], fx)
        rel = [abs(a - b) / b for a, b in zip(losses, ref)]
        out["variants"][name] = {"rounded": sorted(VARIANTS[name]), "losses": losses, "rel": rel,
                                 "max_rel": max(rel)}
        print(f"{name}: max rel {max(rel):.4%} ({time.time() - t0:.0f} s)", flush=True)
        with open(out_path, "w") as f:
            json.dump(out, f, indent=1)


if __name__ == "__main__":
    main(sys.argv[1:] or list(VARIANTS))
