"""ctypes binding of libllmk.so — the C ABI declared in include/llmk.h.

This is the Python-side FFI stub a host program uses to call the sm_100a
kernels (tests and bench.py go through it). It only moves pointers and sizes:
device memory comes from the caller (torch tensors here), and every call
raises LlmkError when the library returns a non-zero status. There is no
fallback: if libllmk.so is missing, importing this module raises.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "libllmk.so")

F32, BF16, F16 = 0, 1, 2
MATH_BF16, MATH_TF32 = 1, 2
EPI_ACCUMULATE, EPI_GELU, EPI_GELU_BWD, EPI_AUX_F32 = 1, 2, 4, 8
ACCUM_DINP, ACCUM_DWEIGHT, ACCUM_DBIAS, ACCUM_DPARAM = 1, 2, 4, 8
DEV_TIMEOUT = 1

STATUS = {0: "ok", 1: "invalid argument", 2: "unsupported", 3: "cuda error", 4: "device wait timed out",
          5: "workspace missing or too small", 6: "nccl error", 7: "no sm_100 device"}


class LlmkError(RuntimeError):
    def __init__(self, fn: str, code: int, detail: str):
        super().__init__(f"{fn} -> {code} ({STATUS.get(code, '?')}): {detail}")
        self.code = code


class Epilogue(C.Structure):
    _fields_ = [("bias", C.c_void_p), ("residual", C.c_void_p), ("ldr", C.c_longlong), ("aux", C.c_void_p),
                ("ldaux", C.c_longlong), ("flags", C.c_int)]


class KernelStat(C.Structure):
    _fields_ = [("name", C.c_char * 24), ("calls", C.c_longlong), ("launches", C.c_longlong), ("ms", C.c_double),
                ("work", C.c_double), ("unit", C.c_int)]


class TrainState(C.Structure):
    _fields_ = [("step", C.c_int), ("world", C.c_int), ("shard_idx", C.c_longlong), ("sample_idx", C.c_longlong)]


class GPT2Config(C.Structure):
    _fields_ = [("max_seq_len", C.c_int), ("vocab_size", C.c_int), ("padded_vocab_size", C.c_int),
                ("num_layers", C.c_int), ("num_heads", C.c_int), ("channels", C.c_int)]


vp, i32, i64, sz, f32, u32p = C.c_void_p, C.c_int, C.c_longlong, C.c_size_t, C.c_float, C.POINTER(C.c_uint)

# name -> (restype, argtypes); restype c_int means "status code, check it".
SIGNATURES: dict[str, tuple] = {
    "llmk_status_string": (C.c_char_p, [i32]),
    "llmk_last_error": (C.c_char_p, []),
    "llmk_version": (C.c_char_p, []),
    "llmk_device_status": (i32, [u32p, i32]),
    "llmk_launch_count": (C.c_ulonglong, []),
    "llmk_gemm_workspace": (sz, [i32, i32, i32, i32]),
    "llmk_gemm": (i32, [vp, i32, i64, vp, i32, i64, vp, i32, i64, i32, i32, i32, i32, C.POINTER(Epilogue), vp, sz,
                        vp]),
    "llmk_matmul_forward": (i32, [vp, i32, vp, vp, vp, i32, i32, i32, i32, vp]),
    "llmk_matmul_backward_workspace": (sz, [i32, i32, i32, i32]),
    "llmk_matmul_backward": (i32, [vp, i32, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp, sz, vp]),
    "llmk_colsum_workspace": (sz, [i32, i32]),
    "llmk_colsum": (i32, [vp, vp, i32, i32, i32, i32, vp, sz, vp]),
    "llmk_colsum_noalloc": (i32, [vp, vp, i32, i32, i32, i32, vp]),
    "llmk_attention_forward": (i32, [vp, i32, vp, vp, i32, i32, i32, i32, i32, vp]),
    "llmk_attention_backward_workspace": (sz, [i32, i32, i32, i32]),
    "llmk_attention_backward": (i32, [vp, vp, vp, i32, vp, i32, vp, i32, i32, i32, i32, vp, sz, vp]),
    "llmk_layernorm_forward": (i32, [vp, i32, vp, vp, vp, vp, vp, i32, i32, vp]),
    "llmk_layernorm_backward_workspace": (sz, [i32, i32]),
    "llmk_layernorm_backward": (i32, [vp, vp, vp, vp, vp, vp, i32, vp, vp, vp, vp, i32, i32, i32, vp, sz, vp]),
    "llmk_gelu_forward": (i32, [vp, vp, i32, i64, vp]),
    "llmk_gelu_backward": (i32, [vp, vp, vp, i32, i64, i32, vp]),
    "llmk_residual_forward": (i32, [vp, vp, vp, i32, i64, vp]),
    "llmk_residual_backward": (i32, [vp, vp, vp, i32, i64, i32, vp]),
    "llmk_cast": (i32, [vp, i32, vp, i32, i64, vp]),
    "llmk_encoder_forward": (i32, [vp, vp, vp, vp, i32, i32, i32, vp]),
    "llmk_encoder_backward_workspace": (sz, [i32, i32]),
    "llmk_encoder_backward": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, vp, sz, vp]),
    "llmk_softmax_crossentropy": (i32, [vp, vp, vp, i32, vp, i32, i32, i32, f32, vp]),
    "llmk_softmax_forward": (i32, [vp, vp, i32, i32, i32, i32, vp]),
    "llmk_crossentropy_forward": (i32, [vp, vp, i32, vp, i32, i32, i32, vp]),
    "llmk_crossentropy_softmax_backward": (i32, [vp, vp, i32, vp, i32, i32, i32, f32, i32, vp]),
    "llmk_matmul_softmax_workspace": (sz, [i32, i32]),
    "llmk_matmul_softmax_forward": (i32, [vp, vp, i32, vp, vp, vp, i32, i32, i32, i32, i32, vp, sz, vp]),
    "llmk_matmul_crossentropy_forward": (i32, [vp, vp, i32, vp, vp, vp, vp, i32, i32, i32, i32, f32, i32, i32, vp, sz,
                                               vp]),
    "llmk_mean": (i32, [vp, vp, i32, vp]),
    "llmk_adamw": (i32, [vp, vp, vp, vp, vp, i64, f32, f32, f32, f32, f32, i32, f32, vp]),
    "llmk_adamw_hparams": (None, [C.POINTER(f32), f32, f32, f32, f32, f32, i32, f32]),
    "llmk_adamw_device_hparams": (i32, [vp, vp, vp, vp, vp, i64, vp, vp]),
    # model (include/llmk_gpt2.h)
    "llmk_gpt2_num_parameters": (sz, [C.POINTER(GPT2Config)]),
    "llmk_gpt2_parameter_count": (sz, [vp]),
    "llmk_gpt2_create": (i32, [C.POINTER(vp), C.POINTER(GPT2Config), i32, i32, i32, vp]),
    "llmk_gpt2_destroy": (i32, [vp]),
    "llmk_gpt2_stream": (i32, [vp, C.POINTER(vp)]),
    "llmk_gpt2_buffers": (i32, [vp, C.POINTER(vp), C.POINTER(vp)]),
    "llmk_gpt2_load_parameters": (i32, [vp, vp, sz]),
    "llmk_gpt2_read_parameters": (i32, [vp, vp, sz]),
    "llmk_gpt2_read_gradients": (i32, [vp, vp, sz]),
    "llmk_gpt2_set_train_data": (i32, [vp, vp, vp]),
    "llmk_gpt2_forward": (i32, [vp, vp, vp]),
    "llmk_gpt2_zero_grad": (i32, [vp]),
    "llmk_gpt2_backward": (i32, [vp]),
    "llmk_gpt2_update": (i32, [vp, f32, f32, f32, f32, f32, i32]),
    "llmk_gpt2_loss": (i32, [vp, C.POINTER(f32)]),
    "llmk_gpt2_device_loss": (i32, [vp, C.POINTER(vp)]),
    "llmk_gpt2_step_device": (i32, [vp, vp, vp, f32, f32, f32, f32, f32, i32]),
    "llmk_gpt2_train_step": (i32, [vp, vp, vp, f32, f32, f32, f32, f32, i32, C.POINTER(f32)]),
    "llmk_gpt2_dp_buckets": (i32, [C.POINTER(GPT2Config), C.POINTER(sz), i32]),
    "llmk_gpt2_to_layer_major": (i32, [C.POINTER(GPT2Config), vp, vp, i32]),
    "llmk_nccl_unique_id": (i32, [vp, sz]),
    "llmk_gpt2_enable_dp": (i32, [vp, vp, sz, i32, i32]),
    "llmk_gpt2_broadcast_parameters": (i32, [vp, i32]),
    "llmk_gpt2_synchronize": (i32, [vp, i32]),
    "llmk_gpt2_set_timing": (i32, [vp, i32]),
    "llmk_gpt2_use_graph": (i32, [vp, i32]),
    "llmk_gpt2_timing_report": (i32, [vp, C.POINTER(KernelStat), i32, C.POINTER(i32)]),
    "llmk_gpt2_get_config": (i32, [vp, C.POINTER(GPT2Config)]),
    "llmk_gpt2_read_optimizer_state": (i32, [vp, vp, vp, sz]),
    "llmk_gpt2_load_optimizer_state": (i32, [vp, vp, vp, sz]),
    "llmk_gpt2_checkpoint_config": (i32, [C.c_char_p, C.POINTER(GPT2Config)]),
    "llmk_gpt2_load_checkpoint": (i32, [vp, C.c_char_p]),
    "llmk_gpt2_save_checkpoint": (i32, [vp, C.c_char_p]),
    "llmk_gpt2_save_state": (i32, [vp, C.c_char_p, C.POINTER(TrainState)]),
    "llmk_gpt2_load_state": (i32, [vp, C.c_char_p, C.POINTER(TrainState)]),
    # include/llmk_data.h
    "llmk_loader_create": (i32, [C.POINTER(vp), C.c_char_p, i32, i32, i32, i32, i32]),
    "llmk_loader_destroy": (i32, [vp]),
    "llmk_loader_next": (i32, [vp, vp, vp]),
    "llmk_loader_reset": (i32, [vp]),
    "llmk_loader_resume": (i32, [vp, sz, sz]),
    "llmk_loader_position": (i32, [vp, C.POINTER(sz), C.POINTER(sz)]),
    "llmk_loader_num_tokens": (i64, [vp]),
}

_lib = None


def lib():
    """Loads libllmk.so once (raises OSError when it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} not built: run `python llm.cpp_b200/build.py`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def check(name: str, rc: int) -> None:
    if rc != 0:
        raise LlmkError(name, rc, lib().llmk_last_error().decode(errors="replace"))


def call(name: str, *args) -> None:
    check(name, getattr(lib(), name)(*args))


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_ptr(stream=None) -> int | None:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def dtype_code(t) -> int:
    import torch
    if t.dtype == torch.bfloat16:
        return BF16
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.float16:
        return F16
    raise TypeError(f"unsupported dtype {t.dtype}")


def device_status(reset: bool = True) -> int:
    v = C.c_uint(0)
    call("llmk_device_status", C.byref(v), 1 if reset else 0)
    return v.value


# ----------------------------------------------------------------- helpers
def gemm(D, A, B, *, a_trans=False, b_trans=False, math=MATH_BF16, bias=None, residual=None, aux=None, flags=0,
         workspace=None, stream=None, M=None, N=None, K=None):
    """D[M,N] = epi(A x B^T); shapes inferred from the storage layouts."""
    if M is None:
        M = A.shape[1] if a_trans else A.shape[0]
    if K is None:
        K = A.shape[0] if a_trans else A.shape[1]
    if N is None:
        N = B.shape[1] if b_trans else B.shape[0]
    ep = Epilogue(ptr(bias), ptr(residual), residual.stride(0) if residual is not None else 0, ptr(aux),
                  aux.stride(0) if aux is not None else 0, flags)
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    call("llmk_gemm", ptr(D), dtype_code(D), D.stride(0), ptr(A), int(a_trans), A.stride(0), ptr(B), int(b_trans),
         B.stride(0), math, M, N, K, C.byref(ep), ptr(workspace), ws_bytes, stream_ptr(stream))


class GPT2:
    """Handle to the native trainer (include/llmk_gpt2.h)."""

    def __init__(self, B: int, T: int, max_seq_len=1024, vocab_size=50257, padded_vocab_size=50304, num_layers=12,
                 num_heads=12, channels=768, math=MATH_BF16, stream=None):
        self.cfg = GPT2Config(max_seq_len, vocab_size, padded_vocab_size, num_layers, num_heads, channels)
        self.B, self.T = B, T
        h = C.c_void_p()
        call("llmk_gpt2_create", C.byref(h), C.byref(self.cfg), B, T, math, stream)
        self.h = h
        self.n = lib().llmk_gpt2_parameter_count(self.h)

    @property
    def stream(self) -> int:
        s = C.c_void_p()
        call("llmk_gpt2_stream", self.h, C.byref(s))
        return s.value

    def buffers(self) -> tuple[int, int]:
        a, b = C.c_void_p(), C.c_void_p()
        call("llmk_gpt2_buffers", self.h, C.byref(a), C.byref(b))
        return a.value, b.value

    def load_parameters(self, params) -> None:
        import numpy as np
        p = np.ascontiguousarray(params, dtype=np.float32)
        assert p.size == self.n, (p.size, self.n)
        call("llmk_gpt2_load_parameters", self.h, p.ctypes.data, p.size)

    def read_parameters(self):
        import numpy as np
        out = np.empty(self.n, np.float32)
        call("llmk_gpt2_read_parameters", self.h, out.ctypes.data, self.n)
        return out

    def read_gradients(self):
        import numpy as np
        out = np.empty(self.n, np.float32)
        call("llmk_gpt2_read_gradients", self.h, out.ctypes.data, self.n)
        return out

    @classmethod
    def from_checkpoint(cls, path: str, B: int, T: int, math=MATH_BF16, stream=None) -> "GPT2":
        """A model shaped by an llm.c v3 model file's header, with its
        parameters loaded (the reference's GPT2(path, B, T) constructor)."""
        c = checkpoint_config(path)
        m = cls(B, T, c.max_seq_len, c.vocab_size, c.padded_vocab_size, c.num_layers, c.num_heads, c.channels,
                math=math, stream=stream)
        m.load_checkpoint(path)
        return m

    def load_checkpoint(self, path: str) -> None:
        call("llmk_gpt2_load_checkpoint", self.h, os.fsencode(path))

    def save_checkpoint(self, path: str) -> None:
        call("llmk_gpt2_save_checkpoint", self.h, os.fsencode(path))

    def save_state(self, path: str, step: int, loader_position=(0, 0), world: int = 1) -> None:
        """Parameters + AdamW moments + step + data-loader position."""
        st = TrainState(step, world, loader_position[0], loader_position[1])
        call("llmk_gpt2_save_state", self.h, os.fsencode(path), C.byref(st))

    def load_state(self, path: str) -> dict:
        st = TrainState()
        call("llmk_gpt2_load_state", self.h, os.fsencode(path), C.byref(st))
        return {"step": st.step, "world": st.world, "loader_position": (st.shard_idx, st.sample_idx)}

    def read_optimizer_state(self):
        import numpy as np
        m, v = np.empty(self.n, np.float32), np.empty(self.n, np.float32)
        call("llmk_gpt2_read_optimizer_state", self.h, m.ctypes.data, v.ctypes.data, self.n)
        return m, v

    def load_optimizer_state(self, m, v) -> None:
        import numpy as np
        m = np.ascontiguousarray(m, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        assert m.size == self.n and v.size == self.n
        call("llmk_gpt2_load_optimizer_state", self.h, m.ctypes.data, v.ctypes.data, self.n)

    def train_step(self, inputs, targets, lr, t, b1=0.9, b2=0.999, eps=1e-8, wd=0.0, want_loss=True):
        """Host tokens in, host loss out (None when want_loss is False)."""
        import numpy as np
        i = np.ascontiguousarray(inputs, dtype=np.int32)
        g = np.ascontiguousarray(targets, dtype=np.int32)
        loss = C.c_float(0.0)
        call("llmk_gpt2_train_step", self.h, i.ctypes.data, g.ctypes.data, lr, b1, b2, eps, wd, t,
             C.byref(loss) if want_loss else None)
        return loss.value if want_loss else None

    def step_device(self, d_inputs: int, d_targets: int, lr, t, b1=0.9, b2=0.999, eps=1e-8, wd=0.0):
        call("llmk_gpt2_step_device", self.h, d_inputs, d_targets, lr, b1, b2, eps, wd, t)

    def forward(self, d_inputs: int, d_targets: int | None):
        call("llmk_gpt2_forward", self.h, d_inputs, d_targets)

    def backward(self):
        call("llmk_gpt2_backward", self.h)

    def update(self, lr, t, b1=0.9, b2=0.999, eps=1e-8, wd=0.0):
        call("llmk_gpt2_update", self.h, lr, b1, b2, eps, wd, t)

    def loss(self) -> float:
        v = C.c_float(0.0)
        call("llmk_gpt2_loss", self.h, C.byref(v))
        return v.value

    def enable_dp(self, unique_id: bytes, rank: int, world: int):
        buf = C.create_string_buffer(bytes(unique_id), len(unique_id))
        call("llmk_gpt2_enable_dp", self.h, C.cast(buf, C.c_void_p), len(unique_id), rank, world)

    def broadcast_parameters(self, root=0):
        call("llmk_gpt2_broadcast_parameters", self.h, root)

    def synchronize(self, timeout_ms=0):
        call("llmk_gpt2_synchronize", self.h, timeout_ms)

    def use_graph(self, enable: bool):
        """Run step_device / train_step as replays of one captured CUDA graph."""
        call("llmk_gpt2_use_graph", self.h, 1 if enable else 0)

    def set_timing(self, enable: bool):
        """Per-kernel-class event timing of later steps (clears old records)."""
        call("llmk_gpt2_set_timing", self.h, 1 if enable else 0)

    def timing_report(self) -> dict:
        """{class: {calls, launches, ms, work, unit}} summed over the timed steps;
        unit is "flop" or "byte" (algorithmic work of the class)."""
        out = (KernelStat * 32)()
        n = C.c_int(0)
        call("llmk_gpt2_timing_report", self.h, out, 32, C.byref(n))
        return {out[i].name.decode(): {"calls": out[i].calls, "launches": out[i].launches, "ms": out[i].ms,
                                       "work": out[i].work, "unit": "flop" if out[i].unit == 0 else "byte"}
                for i in range(min(n.value, 32))}

    def close(self):
        if getattr(self, "h", None):
            lib().llmk_gpt2_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def checkpoint_config(path: str) -> GPT2Config:
    """Configuration in an llm.c v3 model file's header (host only; checks
    magic, version and that the file holds exactly that many parameters)."""
    c = GPT2Config()
    call("llmk_gpt2_checkpoint_config", os.fsencode(path), C.byref(c))
    return c


class DataLoader:
    """Token-shard loader (include/llmk_data.h) with the reference
    DataLoader's constructor arguments and batch order (utils/dataloader.h)."""

    def __init__(self, path: str, B: int, T: int, rank: int = 0, world: int = 1, shuffle: bool = False):
        import numpy as np
        self.B, self.T = B, T
        h = C.c_void_p()
        call("llmk_loader_create", C.byref(h), os.fsencode(path), B, T, rank, world, 1 if shuffle else 0)
        self.h = h
        self.num_tokens = lib().llmk_loader_num_tokens(self.h)
        self.inputs = np.empty((B, T), np.int32)
        self.targets = np.empty((B, T), np.int32)

    def next_batch(self):
        """Fills and returns (inputs, targets), int32 arrays of shape (B, T)
        owned by the loader (overwritten by the next call)."""
        call("llmk_loader_next", self.h, self.inputs.ctypes.data, self.targets.ctypes.data)
        return self.inputs, self.targets

    def reset(self):
        call("llmk_loader_reset", self.h)

    def resume(self, shard_idx: int, sample_idx: int):
        call("llmk_loader_resume", self.h, shard_idx, sample_idx)

    def position(self) -> tuple[int, int]:
        a, b = C.c_size_t(0), C.c_size_t(0)
        call("llmk_loader_position", self.h, C.byref(a), C.byref(b))
        return a.value, b.value

    def close(self):
        if getattr(self, "h", None):
            lib().llmk_loader_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    call("llmk_nccl_unique_id", C.cast(buf, C.c_void_p), 128)
    return buf.raw
