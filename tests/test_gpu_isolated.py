"""The isolated-op workloads on the GPU against their CPU restatements
(oracle/isolated.py), fp32 on the same bf16 inputs.

Tolerances: both kernels return bf16, so one bf16 step of the output scale
(about 0.4% relative) plus the bf16 rounding of intermediate operands the
kernels feed to the tensor cores (the neighbour mean; the softmax weights).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_io import mb
from oracle import isolated as ISO

pytestmark = pytest.mark.gpu
DEV = "cuda"
ops = mb.ops


def _message_case(n_pos, seed, w_std=0.05):
    nbr, _ = mb.hexgraph.message_graph(n_pos, 256, 40, 200, seed=seed)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(nbr.shape[0], 256, generator=g).to(torch.bfloat16)
    w = (torch.randn(256, 256, generator=g) * w_std).to(torch.bfloat16)
    b = torch.randn(256, generator=g) * 0.02
    return x, torch.from_numpy(nbr), w, b


@pytest.mark.parametrize("n_pos,rows", [(8, None), (5, 1000), (3, 37), (160, None)])
def test_hex_message_pass_matches_restatement(n_pos, rows):
    """Against the fp64 restatement: one tile per CTA for the small cases;
    160 positions (40,960 rows, 640 tiles of 64 rows) give each persistent CTA
    four or five tiles, so the window ring's refills, both accumulator
    buffers and the alternating tile barriers all run."""
    x, nbr, w, b = _message_case(n_pos, 7 + n_pos)
    if rows is not None:  # a row count off the 128-row tile, neighbours clipped to it
        x, nbr = x[:rows].contiguous(), nbr[:rows].clone()
        nbr[nbr >= rows] = -1
    want = ISO.hex_message_pass(x.double(), nbr, w.double(), b.double())
    got = ops.hex_message_pass(x.to(DEV), nbr.to(DEV), ops.weight_image(w.to(DEV)), b.to(DEV))
    torch.cuda.synchronize()
    torch.testing.assert_close(got.double().cpu(), want, rtol=1e-2, atol=2e-2)
    mb._lib.check_device_error()


@pytest.mark.parametrize("layout", ["far", "strided"])
def test_hex_message_pass_far_neighbours_and_strided_rows(layout):
    """Neighbours outside a tile's rows +- 64 (read from global memory, not
    the shared-memory window), and strided rows (the gathering row GEMM)."""
    x, nbr, w, b = _message_case(4, 21)
    n = x.shape[0]
    if layout == "far":
        g = torch.Generator().manual_seed(5)
        far = torch.randint(0, n, (n, 6), generator=g, dtype=torch.int32)
        keep = torch.rand(n, 6, generator=g) < 0.3
        nbr = torch.where(keep, far, nbr)
        xd = x.to(DEV)
    else:
        xd = torch.empty(n, 384, dtype=torch.bfloat16, device=DEV)[:, :256]
        xd.copy_(x.to(DEV))
    want = ISO.hex_message_pass(x.double(), nbr, w.double(), b.double())
    got = ops.hex_message_pass(xd, nbr.to(DEV), ops.weight_image(w.to(DEV)), b.to(DEV))
    torch.cuda.synchronize()
    torch.testing.assert_close(got.double().cpu(), want, rtol=1e-2, atol=2e-2)
    mb._lib.check_device_error()


def test_hex_message_pass_edges():
    x, nbr, w, b = _message_case(2, 3)
    nbr[:100] = -1  # rows with no neighbour: y = x + b
    got = ops.hex_message_pass(x.to(DEV), nbr.to(DEV), ops.weight_image(w.to(DEV)), b.to(DEV)).cpu()
    assert torch.equal(got[:100], (x[:100].float() + b).to(torch.bfloat16))
    # W = 0: y = bf16(x + b) everywhere
    got = ops.hex_message_pass(x.to(DEV), nbr.to(DEV), ops.weight_image(torch.zeros_like(w).to(DEV)), b.to(DEV))
    assert torch.equal(got.cpu(), (x.float() + b).to(torch.bfloat16))
    with pytest.raises(ValueError, match="alias"):
        xd = x.to(DEV)
        ops.hex_message_pass(xd, nbr.to(DEV), ops.weight_image(w.to(DEV)), b.to(DEV), out=xd)


def _attention_case(n_pos, heads, seed, layout="phld"):
    coords, valid = mb.hexgraph.attention_layout(n_pos, 256, seed=seed)
    g = torch.Generator().manual_seed(seed)
    shape = (n_pos, heads, 256, 32) if layout == "phld" else (n_pos, 256, heads, 32)
    q, k, v = (torch.randn(*shape, generator=g).to(torch.bfloat16) for _ in range(3))
    if layout != "phld":
        q, k, v = (t.permute(0, 2, 1, 3) for t in (q, k, v))
    bias = torch.randn(33, 33, heads, generator=g) * 0.02
    return q, k, v, torch.from_numpy(coords), torch.from_numpy(valid), bias


@pytest.mark.parametrize("layout", ["phld", "plhd"])
def test_axial_attention_matches_restatement(layout):
    q, k, v, coords, valid, bias = _attention_case(12, 8, 5, layout)
    valid[:4] = torch.tensor([32, 128, 129, 256], dtype=torch.int32)  # tile edges
    want = ISO.axial_attention(q.double(), k.double(), v.double(), coords, valid, bias.double())
    dev = [t.to(DEV) for t in (q, k, v)]
    got = ops.axial_attention(*dev, coords.to(DEV), valid.to(DEV), bias.to(DEV))
    torch.cuda.synchronize()
    torch.testing.assert_close(got.double().cpu(), want, rtol=2e-2, atol=2e-2)
    for p in range(12):
        assert torch.count_nonzero(got[p, :, int(valid[p]):].cpu()) == 0
    mb._lib.check_device_error()


def test_axial_attention_large_bias_and_empty():
    q, k, v, coords, valid, bias = _attention_case(4, 2, 9)
    bias = bias * 100  # the offset bias dominates the dot products
    valid[3] = 0
    want = ISO.axial_attention(q.double(), k.double(), v.double(), coords, valid, bias.double())
    got = ops.axial_attention(q.to(DEV), k.to(DEV), v.to(DEV), coords.to(DEV), valid.to(DEV), bias.to(DEV))
    torch.testing.assert_close(got.double().cpu(), want, rtol=2e-2, atol=2e-2)
    assert torch.count_nonzero(got[3].cpu()) == 0
