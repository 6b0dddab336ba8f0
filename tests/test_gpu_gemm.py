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


# ------------------------------------------------ every projection shape
@pytest.mark.parametrize("k,n", [(256, 128), (256, 384), (256, 512), (256, 768), (256, 1024), (512, 256),
                                 (512, 512), (512, 128), (512, 640)])
@pytest.mark.parametrize("m", [1, 129, 5000, 60000])
def test_copy_prologue_store_shapes(k, n, m):
    """bf16 rows of width K = 256 / 512 times an (N, K) weight, N a multiple
    of 128 (several N blocks on one A tile, a 128-wide last block), with
    bias, ReLU and the fp32 addend; strided input and output rows."""
    g = torch.Generator(device="cpu").manual_seed(m * 7 + k + n)
    xs = torch.randn(m, k + 64, generator=g).to(torch.bfloat16).to(DEV)
    x = xs[:, 32:32 + k]
    w = (torch.randn(n, k, generator=g) / (k ** 0.5)).to(DEV)
    b = torch.randn(n, generator=g).to(DEV)
    add = torch.randn(m, n, generator=g).to(DEV)
    img = ops.weight_image(w)
    ref = x.float() @ w.to(torch.bfloat16).float().t() + b
    out = torch.empty(m, n + 64, dtype=torch.bfloat16, device=DEV)[:, 64:]
    ops.gemm_rows(x, img, bias=b, out=out)
    torch.cuda.synchronize()
    _close(out, ref)
    _close(ops.gemm_rows(x, img, bias=b, relu=True, add=add), (ref + add).relu())
    mb._lib.check_device_error()


@pytest.mark.parametrize("n", [256, 512, 768, 1024])
@pytest.mark.parametrize("m", [3, 4000])
def test_ln_prologue_wide(n, m):
    g = torch.Generator(device="cpu").manual_seed(n + m)
    x = (torch.randn(m, 256, generator=g) * 3 - 1).to(DEV)
    w = (torch.randn(n, 256, generator=g) / 16).to(DEV)
    b = torch.randn(n, generator=g).to(DEV)
    gam, bet = torch.randn(256, generator=g).to(DEV), torch.randn(256, generator=g).to(DEV)
    out = ops.gemm_rows(x, ops.weight_image(w), bias=b, gamma=gam, beta=bet, relu=True)
    z = F.layer_norm(x, (256,), gam, bet).to(torch.bfloat16).float()
    torch.cuda.synchronize()
    _close(out, (z @ w.to(torch.bfloat16).float().t() + b).relu())


@pytest.mark.parametrize("m", [7, 9000])
def test_k512_residual_and_k1024_split(m):
    """residual += a @ W^T + b for K = 512 in one launch and K = 1024 as two
    launches over 512-column slices (the FFN's down-projection)."""
    g = torch.Generator(device="cpu").manual_seed(m)
    a = torch.randn(m, 1024, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(256, 1024, generator=g) / 32).to(DEV)
    b = torch.randn(256, generator=g).to(DEV)
    res0 = torch.randn(m, 256, generator=g).to(DEV)
    res = res0.clone()
    ops.gemm_rows(a[:, :512], ops.weight_image(w[:, :512]), bias=b, residual=res)
    _close(res, res0 + a[:, :512].float() @ w[:, :512].to(torch.bfloat16).float().t() + b)
    ops.gemm_rows(a[:, 512:], ops.weight_image(w[:, 512:]), residual=res)
    torch.cuda.synchronize()
    _close(res, res0 + a.float() @ w.to(torch.bfloat16).float().t() + b)
    mb._lib.check_device_error()


@pytest.mark.parametrize("n,n_out", [(128, 1), (128, 3), (256, 3), (256, 4)])
@pytest.mark.parametrize("m", [1, 130, 20000])
def test_head_epilogue(n, n_out, m):
    """out = relu(x W^T + b + tok[pos]) @ w_out^T + b_out (the decoder head's
    hidden and output layers in one launch) against fp32 torch."""
    g = torch.Generator(device="cpu").manual_seed(n * 11 + n_out + m)
    p = 37
    x = torch.randn(m, 256, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(n, 256, generator=g) / 16).to(DEV)
    b = torch.randn(n, generator=g).to(DEV)
    tok_all = torch.randn(p, 2 * n, generator=g).to(torch.bfloat16).to(DEV)
    tok = tok_all[:, n:]  # strided view, as the engine passes one head's half
    pos = torch.randint(0, p, (m,), generator=g).to(DEV)
    w_out = torch.randn(n_out, n, generator=g).to(DEV) / 8
    b_out = torch.randn(n_out, generator=g).to(DEV)
    got = ops.gemm_head(x, ops.weight_image(w), b, tok, pos, w_out, b_out)
    hid = (x.float() @ w.to(torch.bfloat16).float().t() + b + tok.float()[pos]).relu()
    want = hid @ w_out.t() + b_out
    torch.cuda.synchronize()
    err = (got - want).abs().max().item()
    assert err <= 1e-3 * want.abs().max().item() + 1e-3, err
    mb._lib.check_device_error()


def test_head_refuses_bad_shapes():
    x = torch.zeros(4, 256, dtype=torch.bfloat16, device=DEV)
    img = ops.weight_image(torch.zeros(384, 256, device=DEV))
    tok = torch.zeros(2, 384, dtype=torch.bfloat16, device=DEV)
    pos = torch.zeros(4, dtype=torch.long, device=DEV)
    with pytest.raises(ValueError, match="hidden width"):
        ops.gemm_head(x, img, None, tok, pos, torch.zeros(1, 384, device=DEV), torch.zeros(1, device=DEV))
    with pytest.raises(ValueError):
        ops.weight_image(torch.zeros(200, 256, device=DEV))
