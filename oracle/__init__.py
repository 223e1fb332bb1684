"""ctypes access to the CPU checkers (TEST INFRASTRUCTURE ONLY).

`orc` wraps liboracle.so (oracle.c, the C restatement of the reference CPU
path); `ref` wraps _ref/libref.so (the reference's own CPU sources). Only
tests/, __graft_entry__.smoke() and bench.py's CPU legs import this module;
the product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libref.so")          # -march=x86-64-v3
REF_LIB_V4 = os.path.join(HERE, "_ref", "libref_v4.so")    # -march=x86-64-v4 (AVX-512)
_AVX512 = ("avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl")


def _host_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    flags = set(line.split(":", 1)[1].split())
                    return all(x in flags for x in _AVX512)
    except OSError:
        pass
    return False


def ref_path() -> str:
    """The reference build for this host: the AVX-512 one when the CPU has it."""
    if os.path.exists(REF_LIB_V4) and _host_has_avx512():
        return REF_LIB_V4
    return REF_LIB


def ref_build() -> str:
    """Compiler flags of the reference build ref() loads."""
    isa = "-march=x86-64-v4" if ref_path() == REF_LIB_V4 else "-march=x86-64-v3"
    return f"g++ -O3 {isa} -ffast-math -fopenmp (CMakeLists.txt Release flags, ISA level of the host)"

fp = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
ip = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
vp, i32, sz, f32, u64 = C.c_void_p, C.c_int, C.c_size_t, C.c_float, C.c_uint64


class Config(C.Structure):
    _fields_ = [("max_seq_len", C.c_int), ("vocab_size", C.c_int), ("padded_vocab_size", C.c_int),
                ("num_layers", C.c_int), ("num_heads", C.c_int), ("channels", C.c_int)]


GPT2_124M = dict(max_seq_len=1024, vocab_size=50257, padded_vocab_size=50304, num_layers=12, num_heads=12,
                 channels=768)

_ORC_SIGS = {
    "orc_fill_normal": (None, [fp, sz, f32, u64, u64]),
    "orc_fill_tokens": (None, [ip, sz, i32, u64, u64]),
    "orc_matmul_forward": (None, [fp, fp, fp, vp, i32, i32, i32]),
    "orc_matmul_backward": (None, [fp, fp, vp, fp, fp, fp, i32, i32, i32]),
    "orc_attention_forward": (None, [fp, fp, vp, fp, i32, i32, i32, i32]),
    "orc_attention_backward": (None, [fp, fp, fp, fp, i32, i32, i32, i32]),
    "orc_layernorm_forward": (None, [fp, vp, vp, fp, fp, fp, i32, i32]),
    "orc_layernorm_backward": (None, [fp, fp, fp, fp, fp, fp, fp, fp, i32, i32]),
    "orc_gelu_forward": (None, [fp, fp, sz]),
    "orc_gelu_backward": (None, [fp, fp, fp, sz]),
    "orc_residual_forward": (None, [fp, fp, fp, sz]),
    "orc_softmax": (None, [fp, fp, i32, i32, i32]),
    "orc_cross_entropy": (f32, [vp, fp, ip, i32, i32]),
    "orc_cross_entropy_softmax_backward": (None, [fp, fp, ip, i32, i32, i32]),
    "orc_encoder_forward": (None, [fp, ip, fp, fp, i32, i32, i32]),
    "orc_encoder_backward": (None, [fp, fp, fp, ip, i32, i32, i32]),
    "orc_adamw": (None, [fp, fp, fp, fp, sz, f32, f32, f32, f32, f32, i32]),
    "orc_gpt2_param_sizes": (sz, [C.POINTER(Config), C.POINTER(C.c_size_t)]),
    "orc_gpt2_init_params": (None, [fp, C.POINTER(Config), u64]),
    "orc_gpt2_create": (vp, [C.POINTER(Config), fp, i32, i32]),
    "orc_gpt2_free": (None, [vp]),
    "orc_gpt2_forward": (f32, [vp, ip, ip]),
    "orc_gpt2_zero_grad": (None, [vp]),
    "orc_gpt2_backward": (None, [vp]),
    "orc_gpt2_update": (None, [vp, f32, f32, f32, f32, f32, i32]),
    "orc_gpt2_params": (C.POINTER(C.c_float), [vp]),
    "orc_gpt2_grads": (C.POINTER(C.c_float), [vp]),
    "orc_gpt2_num_params": (sz, [vp]),
    "orc_gpt2_activation": (C.POINTER(C.c_float), [vp, C.c_char_p]),
}

_REF_SIGS = {
    "ref_matmul_forward": (None, [fp, fp, fp, vp, i32, i32, i32, i32]),
    "ref_matmul_backward": (None, [fp, fp, fp, fp, fp, fp, i32, i32, i32, i32]),
    "ref_attention_forward": (None, [fp, vp, fp, i32, i32, i32, i32]),
    "ref_attention_backward": (None, [fp, fp, fp, i32, i32, i32, i32]),
    "ref_layernorm_forward": (None, [fp, fp, fp, fp, fp, fp, i32, i32, i32]),
    "ref_layernorm_backward": (None, [fp, fp, fp, fp, fp, fp, fp, i32, i32, i32]),
    "ref_gelu_forward": (None, [fp, fp, i32, i32, i32]),
    "ref_gelu_backward": (None, [fp, fp, fp, i32, i32, i32]),
    "ref_gpt2_train": (i32, [C.c_char_p, i32, i32, ip, ip, i32, f32, fp, np.ctypeslib.ndpointer(dtype=np.float64)]),
    "ref_loader_create": (vp, [C.c_char_p, i32, i32, i32, i32, i32]),
    "ref_loader_destroy": (None, [vp]),
    "ref_loader_next": (None, [vp, ip, ip]),
    "ref_loader_reset": (None, [vp]),
    "ref_loader_resume": (None, [vp, sz, sz]),
    "ref_loader_num_tokens": (C.c_longlong, [vp]),
}


def _load(path, sigs):
    L = C.CDLL(path)
    for n, (res, args) in sigs.items():
        f = getattr(L, n)
        f.restype = res
        f.argtypes = args
    return L


_orc = None
_ref = None


def build_oracle() -> None:
    if not os.path.exists(ORACLE_LIB):
        subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)


def orc():
    """liboracle.so (built on demand with gcc: the build needs no reference tree)."""
    global _orc
    if _orc is None:
        build_oracle()
        _orc = _load(ORACLE_LIB, _ORC_SIGS)
    return _orc


def ref_available() -> bool:
    return os.path.exists(ref_path())


def ref():
    global _ref
    if _ref is None:
        if not ref_available():
            raise OSError(f"{REF_LIB} not built (run `make -C oracle ref REF=<reference root>` where the "
                          f"reference tree exists)")
        _ref = _load(ref_path(), _REF_SIGS)
    return _ref


def f32a(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


def normal(shape, seed, stream=2, std=1.0) -> np.ndarray:
    out = np.empty(int(np.prod(shape)), dtype=np.float32)
    orc().orc_fill_normal(out, out.size, std, seed, stream)
    return out.reshape(shape)


def tokens(n, vocab, seed, stream=1) -> np.ndarray:
    out = np.empty(n, dtype=np.int32)
    orc().orc_fill_tokens(out, n, vocab, seed, stream)
    return out


def config(**kw) -> Config:
    d = dict(GPT2_124M)
    d.update(kw)
    return Config(**d)


def param_sizes(cfg: Config) -> list[int]:
    arr = (C.c_size_t * 16)()
    orc().orc_gpt2_param_sizes(C.byref(cfg), arr)
    return list(arr)


def init_params(cfg: Config, seed: int) -> np.ndarray:
    n = sum(param_sizes(cfg))
    p = np.empty(n, dtype=np.float32)
    orc().orc_gpt2_init_params(p, C.byref(cfg), seed)
    return p


def write_checkpoint(path: str, cfg: Config, params: np.ndarray) -> None:
    """llm.c v3 checkpoint in the order gpt2/gpt2.cpp:112-230 reads it."""
    header = np.zeros(256, dtype=np.int32)
    header[:8] = [20240326, 3, cfg.max_seq_len, cfg.vocab_size, cfg.num_layers, cfg.num_heads, cfg.channels,
                  cfg.padded_vocab_size]
    with open(path, "wb") as f:
        f.write(header.tobytes())
        f.write(f32a(params).tobytes())


class Model:
    """The oracle GPT-2 (fp32, CPU)."""

    def __init__(self, cfg: Config, params: np.ndarray, B: int, T: int):
        self.cfg, self.B, self.T = cfg, B, T
        self._p = f32a(params)
        self.h = orc().orc_gpt2_create(C.byref(cfg), self._p, B, T)
        self.n = orc().orc_gpt2_num_params(self.h)

    def forward(self, inputs, targets) -> float:
        return orc().orc_gpt2_forward(self.h, np.ascontiguousarray(inputs, dtype=np.int32),
                                      np.ascontiguousarray(targets, dtype=np.int32))

    def zero_grad(self):
        orc().orc_gpt2_zero_grad(self.h)

    def backward(self):
        orc().orc_gpt2_backward(self.h)

    def update(self, lr, b1=0.9, b2=0.999, eps=1e-8, wd=0.0, t=1):
        orc().orc_gpt2_update(self.h, lr, b1, b2, eps, wd, t)

    def params(self) -> np.ndarray:
        return np.ctypeslib.as_array(orc().orc_gpt2_params(self.h), shape=(self.n,)).copy()

    def grads(self) -> np.ndarray:
        return np.ctypeslib.as_array(orc().orc_gpt2_grads(self.h), shape=(self.n,)).copy()

    def activation(self, name: str, shape) -> np.ndarray:
        p = orc().orc_gpt2_activation(self.h, name.encode())
        return np.ctypeslib.as_array(p, shape=(int(np.prod(shape)),)).reshape(shape).copy()

    def __del__(self):
        try:
            orc().orc_gpt2_free(self.h)
        except Exception:
            pass
