"""tcgen05 fused row GEMM (LayerNorm prologue / bias / ReLU / residual
epilogue) against an fp32 torch reference on the same bf16 operands.
Tolerance: one bf16 rounding of the output plus fp32 summation order,
|err| <= 1e-2 * max|ref| + 1e-3."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from golden_io import mb

pytestmark = pytest.mark.gpu
ops = mb.ops
DEV = "cuda"


def _close(got, want):
    err = (got.float() - want).abs().max().item()
    assert err <= 1e-2 * want.abs().max().item() + 1e-3, err


@pytest.mark.parametrize("m", [1, 127, 128, 129, 1000, 40000])
def test_ln_prologue_store(m):
    g = torch.Generator(device="cpu").manual_seed(m)
    x = (torch.randn(m, 256, generator=g) * 2 + 0.5).to(DEV)
    w = (torch.randn(256, 256, generator=g) / 16).to(DEV)
    b = torch.randn(256, generator=g).to(DEV)
    gam, bet = torch.randn(256, generator=g).to(DEV), torch.randn(256, generator=g).to(DEV)
    img = ops.weight_image(w)
    out = ops.gemm_rows(x, img, bias=b, gamma=gam, beta=bet)
    z = F.layer_norm(x, (256,), gam, bet).to(torch.bfloat16).float()
    want = z @ w.to(torch.bfloat16).float().t() + b
    torch.cuda.synchronize()
    _close(out, want)
    relu = ops.gemm_rows(x, img, bias=b, gamma=gam, beta=bet, relu=True)
    _close(relu, want.relu())
    mb._lib.check_device_error()


@pytest.mark.parametrize("m", [5, 128, 3333, 70000])
def test_copy_prologue_residual(m):
    g = torch.Generator(device="cpu").manual_seed(7 + m)
    a = torch.randn(m, 256, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(256, 256, generator=g) / 16).to(DEV)
    b = torch.randn(256, generator=g).to(DEV)
    res0 = torch.randn(m, 256, generator=g).to(DEV)
    res = res0.clone()
    ops.gemm_rows(a, ops.weight_image(w), bias=b, residual=res)
    want = res0 + a.float() @ w.to(torch.bfloat16).float().t() + b
    torch.cuda.synchronize()
    _close(res, want)
    mb._lib.check_device_error()


def test_strided_output_and_no_bias():
    m = 777
    x = torch.randn(m, 256, device=DEV)
    w = torch.randn(256, 256, device=DEV) / 16
    gam, bet = torch.ones(256, device=DEV), torch.zeros(256, device=DEV)
    buf = torch.zeros(m, 512, dtype=torch.bfloat16, device=DEV)
    ops.gemm_rows(x, ops.weight_image(w), gamma=gam, beta=bet, out=buf[:, 256:])
    want = F.layer_norm(x, (256,)).to(torch.bfloat16).float() @ w.to(torch.bfloat16).float().t()
    _close(buf[:, 256:], want)
    assert torch.count_nonzero(buf[:, :256]) == 0


@pytest.mark.parametrize("m", [1, 129, 1000, 40000])
@pytest.mark.parametrize("n_ln", [1, 2, 3])
def test_residual_layernorm_epilogue(m, n_ln):
    """x += a W^T + b and up to three LayerNorms of the updated rows (bf16
    destinations, one of them a column view) from one launch."""
    g = torch.Generator(device="cpu").manual_seed(m + n_ln)
    a = torch.randn(m, 256, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(256, 256, generator=g) / 16).to(DEV).to(torch.bfloat16)
    b = torch.randn(256, generator=g).to(DEV)
    x = (torch.randn(m, 256, generator=g) * 3 + 1).to(DEV)
    want_x = x + a.float() @ w.float().t() + b
    lns, outs = [], []
    wide = torch.empty(m, 512, dtype=torch.bfloat16, device=DEV)
    for j in range(n_ln):
        gam = torch.randn(256, generator=g).to(DEV)
        bet = torch.randn(256, generator=g).to(DEV)
        o = wide[:, 256:] if j == 0 else torch.empty(m, 256, dtype=torch.bfloat16, device=DEV)
        lns.append((gam, bet, o))
    ops.gemm_rows_ln(a, ops.weight_image(w), b, x, lns)
    torch.cuda.synchronize()
    torch.testing.assert_close(x, want_x, rtol=1e-4, atol=1e-3)
    for gam, bet, o in lns:
        want = F.layer_norm(want_x, (256,), gam, bet)
        tol = 2e-2
        torch.testing.assert_close(o.float(), want, rtol=tol, atol=tol * max(1.0, want.abs().max().item()) / 4)
    mb._lib.check_device_error()


@pytest.mark.gpu
def test_residual_layernorm_rejects_fp32_outputs():
    """The fused epilogue stages bf16 row segments only: an fp32 LayerNorm
    destination is refused before launch (the caller takes the unfused path)."""
    a = torch.zeros(64, 256, dtype=torch.bfloat16, device=DEV)
    x = torch.zeros(64, 256, device=DEV)
    w = ops.weight_image(torch.zeros(256, 256, device=DEV))
    one, zero = torch.ones(256, device=DEV), torch.zeros(256, device=DEV)
    with pytest.raises(ValueError):
        ops.gemm_rows_ln(a, w, None, x, [(one, zero, torch.empty(64, 256, device=DEV))])
