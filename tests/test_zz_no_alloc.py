"""llmk_colsum_noalloc: the column-sum entry point that allocates nothing.

It exists for callers that may not allocate device memory at call time
(code inside another framework's memory pool or under a fixed memory budget,
or code that must not stall its stream on cudaMalloc). Its partial sums live
in a fixed array inside the library instead of a caller workspace. This test
calls it through the C ABI twice in a row, with different shapes, dtypes and
accumulate modes, and checks each result against llmk_colsum (the entry
point with a caller workspace) at the tolerance of the other fp32 bandwidth
kernels. The file sorts last so that a stop-at-first-failure run has already
run every other test; it also passes alone in a fresh process.
"""
import numpy as np
import pytest

import oracle as O
from conftest import max_rel_err

pytestmark = pytest.mark.gpu


def _colsum_with_workspace(llmk, torch, x, M, N, accumulate, init):
    out = init.clone()
    wsb = llmk.lib().llmk_colsum_workspace(M, N)
    ws = torch.empty(wsb // 4 + 64, device=x.device)
    llmk.call("llmk_colsum", out.data_ptr(), x.data_ptr(), llmk.dtype_code(x), M, N, accumulate, ws.data_ptr(), wsb,
              llmk.stream_ptr())
    return out


def test_colsum_noalloc_matches_workspace_version(cuda_dev):
    import torch
    import llmk
    cases = [  # (M, N, dtype, accumulate)
        (16384, 2304, torch.bfloat16, 0),
        (1000, 768, torch.float32, 1),
    ]
    for i, (M, N, dt, acc) in enumerate(cases):
        x = torch.from_numpy(O.normal((M, N), 900 + i)).to(cuda_dev).to(dt)
        init = torch.from_numpy(O.normal((N,), 950 + i)).to(cuda_dev)
        ref = _colsum_with_workspace(llmk, torch, x, M, N, acc, init)
        out = init.clone()
        llmk.call("llmk_colsum_noalloc", out.data_ptr(), x.data_ptr(), llmk.dtype_code(x), M, N, acc,
                  llmk.stream_ptr())
        torch.cuda.synchronize()
        assert max_rel_err(out, ref) < 1e-5, (i, max_rel_err(out, ref))
    assert llmk.device_status() == 0


def test_colsum_noalloc_rejects_oversized(cuda_dev):
    import torch
    import llmk
    N = 300000  # one chunk of N floats already exceeds the fixed scratch
    x = torch.zeros(64, N, device=cuda_dev)
    out = torch.zeros(N, device=cuda_dev)
    with pytest.raises(llmk.LlmkError) as e:
        llmk.call("llmk_colsum_noalloc", out.data_ptr(), x.data_ptr(), llmk.F32, 64, N, 0, llmk.stream_ptr())
    assert e.value.code == 2
    assert "scratch" in str(e.value)
