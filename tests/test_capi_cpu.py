"""C ABI checks that need no GPU: the library loads, every function declared
in include/*.h is exported, argument validation fails cleanly, and the
host-only planning helpers (workspace sizes, DP buckets, parameter layout)
are consistent."""
import ctypes as C
import glob
import os
import re

import numpy as np
import pytest

import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for h in sorted(glob.glob(os.path.join(ROOT, "include", "*.h"))):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(llmk_\w+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_every_declared_symbol_is_exported(llmk_lib):
    import llmk
    decl = declared_functions()
    assert len(decl) >= 40, decl
    L = C.CDLL(llmk.LIB_PATH)
    missing = [n for n in decl if not hasattr(L, n)]
    assert not missing, missing
    # and the Python FFI stub binds every one of them
    assert sorted(set(decl) - set(llmk.exported_symbols())) == []


def test_argument_validation_without_gpu(llmk_lib):
    import llmk
    L = llmk.lib()
    assert L.llmk_gemm(None, 0, 0, None, 0, 0, None, 0, 0, llmk.MATH_BF16, 1, 1, 1, None, None, 0, None) == 1
    assert L.llmk_attention_forward(None, llmk.BF16, None, None, llmk.BF16, 1, 64, 192, 1, None) == 1
    assert b"null" in L.llmk_last_error()
    assert L.llmk_status_string(4) == b"device wait timed out"
    assert L.llmk_matmul_backward_workspace(8192, 768, 2304, llmk.MATH_BF16) > 0
    # D (fp32 per row and head) | fp32 dQ accumulator | bf16 copy of dO
    assert L.llmk_attention_backward_workspace(8, 1024, 2304, 12) == 8 * 12 * 1024 * 4 + 8 * 1024 * 768 * (4 + 2)
    assert L.llmk_layernorm_backward_workspace(16384, 768) > 0
    # fused lm_head: one (max, sum) pair per row and 64-column slot, then the row lse
    assert L.llmk_matmul_softmax_workspace(8192, 50304) == 8192 * 786 * 8 + 8192 * 4  # + one lse per row
    assert L.llmk_matmul_crossentropy_forward(None, None, llmk.BF16, None, None, None, None, 8, 64, 512, 500, 1.0, 1,
                                              llmk.MATH_BF16, None, 0, None) == 1
    fake = 1 << 20  # never dereferenced: the missing workspace is refused first
    assert L.llmk_matmul_crossentropy_forward(fake, fake, llmk.BF16, fake, fake, None, fake, 8, 64, 512, 500, 1.0, 1,
                                              llmk.MATH_BF16, None, 0, None) == 5
    assert L.llmk_matmul_softmax_forward(fake, fake, llmk.BF16, fake, fake, None, 8, 64, 510, 500, llmk.MATH_BF16,
                                         fake, 1 << 20, None) == 2  # Vp % 8
    # the column sums read fp32 or bf16 only: fp16 is refused, not read as fp32
    assert L.llmk_colsum(fake, fake, llmk.F16, 64, 64, 0, fake, 1 << 20, None) == 2
    assert b"fp32 or bf16" in L.llmk_last_error()
    assert L.llmk_colsum_noalloc(fake, fake, llmk.F16, 64, 64, 0, None) == 2
    assert L.llmk_colsum_noalloc(fake, fake, 7, 64, 64, 0, None) == 2
    # the no-allocation column sum accepts up to 262144 columns, refused above before any device call
    assert L.llmk_colsum_noalloc(fake, fake, llmk.F32, 64, (1 << 18) + 8, 0, None) == 2
    assert b"exceeds the fixed scratch" in L.llmk_last_error()


def test_dp_buckets_partition_parameters(llmk_lib):
    import llmk
    cfg = llmk.GPT2Config(1024, 50257, 50304, 12, 12, 768)
    n = llmk.lib().llmk_gpt2_dp_buckets(C.byref(cfg), None, 0)
    assert n == 14
    arr = (C.c_size_t * (2 * n))()
    assert llmk.lib().llmk_gpt2_dp_buckets(C.byref(cfg), arr, n) == n
    ranges = sorted((arr[2 * i], arr[2 * i + 1]) for i in range(n))
    total = llmk.lib().llmk_gpt2_num_parameters(C.byref(cfg))
    assert total == 124475904
    pos = 0
    for b, e in ranges:
        assert b == pos and e > b
        pos = e
    assert pos == total


def test_layer_major_permutation_roundtrip(llmk_lib):
    import llmk
    cfgo = O.config(max_seq_len=64, vocab_size=100, padded_vocab_size=128, num_layers=3, num_heads=2, channels=128)
    cfg = llmk.GPT2Config(64, 100, 128, 3, 2, 128)
    n = llmk.lib().llmk_gpt2_num_parameters(C.byref(cfg))
    assert n == sum(O.param_sizes(cfgo))
    src = np.arange(n, dtype=np.float32)
    lm = np.empty_like(src)
    back = np.empty_like(src)
    llmk.call("llmk_gpt2_to_layer_major", C.byref(cfg), src.ctypes.data, lm.ctypes.data, 0)
    llmk.call("llmk_gpt2_to_layer_major", C.byref(cfg), lm.ctypes.data, back.ctypes.data, 1)
    assert np.array_equal(back, src)
    assert not np.array_equal(lm, src)
    assert np.array_equal(np.sort(lm), src)


def test_dataloader_adapter_matches_reference_api(llmk_lib, tmp_path):
    """include/llmk_dataloader.hpp (the reference's DataLoader class over the
    C ABI) compiles, links, and its NextBatch overloads return the batches the
    shard holds; a bad shard throws std::invalid_argument."""
    import shutil
    import subprocess
    import llmk
    from oracle import dataloader as D
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    toks = np.arange(1, 2 * 3 * 16 + 2) % 50000
    D.write_shard(str(tmp_path / "a.bin"), toks)
    (tmp_path / "bad.bin").write_bytes(b"\0" * 1100)
    src = tmp_path / "loader.cpp"
    src.write_text(r'''
#include <cstdio>
#include "llmk_dataloader.hpp"
int main(int argc, char** argv) {
  DataLoader dl(argv[1], 2, 16, 0, 1, false);
  std::vector<int> in(32), tg(32);
  dl.NextBatch(in, tg);
  int in2[32], tg2[32];
  dl.NextBatch(in2, tg2);
  std::printf("%zu %d %d %d %d\n", dl.num_tokens, in[0], tg[31], in2[0], tg2[31]);
  try { std::vector<int> bad(3); dl.NextBatch(bad, tg); return 2; } catch (const std::invalid_argument&) {}
  try { DataLoader b(argv[2], 2, 16, 0, 1, false); return 3; } catch (const std::invalid_argument&) {}
  return 0;
}
''')
    exe = tmp_path / "loader"
    lib_dir = os.path.dirname(llmk.LIB_PATH)
    r = subprocess.run([gxx, "-std=c++17", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe),
                        "-L", lib_dir, "-l:libllmk.so", f"-Wl,-rpath,{lib_dir}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe), str(tmp_path / "a.bin"), str(tmp_path / "bad.bin")], capture_output=True,
                       text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.split() == [str(toks.size), "1", "33", "33", "65"]


def test_adapter_compiles_and_links(llmk_lib, tmp_path):
    """include/llmk_gpt2cuda.hpp (the reference's gpt2cuda:: API over the C ABI),
    header-only use: every op compiles against a DevVecf-like type and links
    against libllmk.so; without a GPU (or with null buffers) each op throws
    the reference's exception types instead of crashing or allocating."""
    import shutil
    import subprocess
    import llmk
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    src = tmp_path / "adapter.cpp"
    src.write_text(r'''
#include <functional>
#include "llmk_gpt2cuda.hpp"
struct DevVecf { float* p = nullptr; size_t n = 0; float* data() const { return p; } size_t size() const { return n; } };
struct DevVeci { int* p = nullptr; size_t n = 0; int* data() const { return p; } size_t size() const { return n; } };
int main() {
  DevVecf a, b, c, d, e, g; DevVeci t; cudaStream_t s = nullptr;
  float h[64] = {};
  std::function<void()> ops[] = {
    [&] { gpt2cuda::BatchMatmulNTForward(a, b, c, d, 1, 1, 8, 8, s); },
    [&] { gpt2cuda::BatchMatmulNTBackward(a, b, c, d, e, g, 1, 1, 8, 8, s); },
    [&] { gpt2cuda::BatchCausalAttentionForward(a, b, c, 1, 64, 192, 1, s); },
    [&] { gpt2cuda::BatchCausalAttentionBackward(a, b, c, d, e, g, 1, 64, 192, 1, s); },
    [&] { gpt2cuda::BatchLayerNormForward(a, b, c, d, e, g, 1, 1, 8, s); },
    [&] { gpt2cuda::BatchLayerNormBackward(a, b, c, d, e, g, b, c, 1, 1, 8, s); },
    [&] { gpt2cuda::BatchGeluForward(a, b, 1, 1, 8, s); },
    [&] { gpt2cuda::BatchGeluBackward(a, b, c, 1, 1, 8, s); },
    [&] { gpt2cuda::BatchResidualForward(a, b, c, 1, 1, 8, s); },
    [&] { gpt2cuda::BatchResidualBackward(a, b, c, 1, 1, 8, s); },
    [&] { gpt2cuda::BatchEncoderForward(a, t, b, c, 1, 1, 8, 8, 8, s); },
    [&] { gpt2cuda::BatchEncoderBackward(a, b, c, t, 1, 1, 8, 8, 8, s); },
    [&] { gpt2cuda::BatchSoftmaxForward(a, b, 1, 1, 8, 8, s); },
    [&] { gpt2cuda::BatchCrossEntropyForward(a, b, t, 1, 1, 8, s); },
    [&] { gpt2cuda::BatchCrossEntropySoftmaxBackward(a, b, t, 1, 1, 8, 8, 1.f, s); },
    [&] { gpt2cuda::BatchMatmulNTSoftmaxForward(a, b, c, d, e, g, 1, 1, 8, 8, 8, s); },
    [&] { gpt2cuda::AdamW(a, b, c, d, 8, gpt2cuda::AdamWConfig{1e-3f, .9f, .999f, 1e-8f, 0.f, 1}, s); },
    [&] { gpt2cuda::LlmkSetWorkspace(nullptr, 0); },
    [&] { gpt2cuda::BatchMatmulNTForward(h, h, h, nullptr, 1, 1, 8, 8); },
    [&] { gpt2cuda::BatchCausalAttentionForward(h, h, h, 1, 1, 192, 1); },
  };
  int thrown = 0;
  for (auto& op : ops) {
    try { op(); } catch (const std::invalid_argument&) { ++thrown; } catch (const std::runtime_error&) { ++thrown; }
  }
  gpt2cuda::BatchSoftmaxBackward(a, b, c, 1, 1, 8, 8, s);  // a no-op, as in the reference
  std::printf("%d %zu\n", thrown, gpt2cuda::GetMatmulSoftmaxWorkSpaceSize(4, 64, 50304));
  return 0;
}
''')
    exe = tmp_path / "adapter"
    lib_dir = os.path.dirname(llmk.LIB_PATH)
    r = subprocess.run([gxx, "-std=c++17", "-I", os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include",
                        str(src), "-o", str(exe), "-L", lib_dir, "-l:libllmk.so", f"-Wl,-rpath,{lib_dir}",
                        "-L", "/usr/local/cuda/lib64", "-lcudart"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    thrown, ws = r.stdout.split()
    # every op but the workspace registration (which needs a device) rejects null buffers / a missing GPU
    assert int(thrown) >= 19, r.stdout
    assert int(ws) == (llmk.lib().llmk_matmul_softmax_workspace(256, 50304) + 3) // 4


def test_dropin_links_against_reference_sources():
    """Link-level drop-in: the reference's own gpt2/cuda/gpt2cuda.cu and
    layer.cu, compiled unchanged from the reference tree, link against
    llm.cpp_b200/dropin/gpt2cuda_llmk.cu + libllmk.so with no undefined symbol
    (the Makefile links once with --no-undefined). Needs the reference tree."""
    import subprocess
    sys_path = os.path.join(ROOT, "__graft_entry__.py")
    assert os.path.exists(sys_path)
    import importlib.util
    spec = importlib.util.spec_from_file_location("graft_entry", sys_path)
    ge = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ge)
    ref = ge.reference_root()
    if ref is None:
        pytest.skip("reference tree not present")
    r = subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "dropin", f"REF={ref}"],
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    lib = os.path.join(ROOT, "oracle", "_ref", "libgpt2cuda_llmk.so")
    nm = subprocess.run(["nm", "-C", "--undefined-only", lib], capture_output=True, text=True).stdout
    assert "gpt2cuda::" not in nm, [ln for ln in nm.splitlines() if "gpt2cuda::" in ln]
