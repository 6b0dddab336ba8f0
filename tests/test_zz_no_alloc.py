"""The allocation-free relay cell pass (mb_cell_pass_noalloc) against the
allocating entry point (mb_cell_pass with a caller scratch buffer).

Some hosts cannot let the library allocate device memory — a runtime that
owns every device buffer, a process under a fixed memory budget — so the
library offers this variant whose scratch is an array compiled into it. The
test drives both through the C ABI on the same inputs, twice in a row (the
fixed array keeps the previous call's contents), and checks the size limit.
Tolerance: both run the same kernels, so 1e-5 absolute / relative.
This file is collected last so that a run stopping at the first failure has
run every other test; it also passes alone in a fresh process.
"""

from __future__ import annotations

import pytest
import torch

import golden_io
from golden_io import mb

pytestmark = pytest.mark.gpu
DEV = "cuda"
_lib = mb._lib


def _noalloc(x, emb, b, out):
    n_cov = b.relay_cell_ptr.numel() - 1
    _lib.call("mb_cell_pass_noalloc", x.data_ptr(), _lib.dtype_code(x.dtype), x.shape[0], emb.data_ptr(),
              emb.shape[0], b.relay_cell_ptr.data_ptr(), n_cov, b.relay_window.data_ptr(), b.relay_class.data_ptr(),
              b.relay_win_ptr.data_ptr(), b.relay_wcell.data_ptr(), x.shape[1], out.data_ptr(),
              _lib.dtype_code(out.dtype), _lib.stream_of(x.device))
    return out


def _alloc(x, emb, b, out):
    n_cov = b.relay_cell_ptr.numel() - 1
    scratch = torch.empty(max(n_cov, 1), x.shape[1], dtype=torch.float32, device=x.device)
    _lib.call("mb_cell_pass", x.data_ptr(), _lib.dtype_code(x.dtype), x.shape[0], emb.data_ptr(), emb.shape[0],
              b.relay_cell_ptr.data_ptr(), n_cov, b.relay_window.data_ptr(), b.relay_class.data_ptr(),
              b.relay_win_ptr.data_ptr(), b.relay_wcell.data_ptr(), x.shape[1], scratch.data_ptr(), out.data_ptr(),
              _lib.dtype_code(out.dtype), _lib.stream_of(x.device))
    return out


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_cell_pass_matches_allocating_entry_point(dtype):
    _lib.load()
    _, _, batch, _, _ = golden_io.forward_case("default")
    b = batch.to(DEV)
    g = torch.Generator().manual_seed(31)
    emb = torch.randn(726, 32, generator=g).to(DEV)
    for call in range(2):  # the second call runs on the array the first one left behind
        x = torch.randn(batch.n_windows, 32, generator=g).to(dtype).to(DEV)
        want = _alloc(x, emb, b, torch.empty_like(x))
        got = _noalloc(x, emb, b, torch.full_like(x, float("nan")))
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float(), want.float(), rtol=1e-5, atol=1e-5, msg=f"call {call}")
    _lib.check_device_error()


def test_noalloc_cell_pass_refuses_sizes_beyond_its_buffer():
    _lib.load()
    _, _, batch, _, _ = golden_io.forward_case("default")
    b = batch.to(DEV)
    h = 4096  # n_cov * h exceeds the 4,194,304-float buffer for this batch
    assert (b.relay_cell_ptr.numel() - 1) * h > 4 * 1024 * 1024
    x = torch.zeros(batch.n_windows, h, device=DEV)
    emb = torch.zeros(726, h, device=DEV)
    with pytest.raises(ValueError, match="fixed buffer"):
        _noalloc(x, emb, b, torch.empty_like(x))
