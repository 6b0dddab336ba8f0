"""Backward kernels against torch autograd of plain differentiable
restatements of each op (fp32 inputs, 1e-4 relative), the reference's
backward test pattern (tests/test_attention_kernel.py:127-254); and
determinism: two runs give identical bits (no atomics)."""

from __future__ import annotations

import pytest
import torch

from golden_io import mb

pytestmark = pytest.mark.gpu
ops = mb.ops
DEV = "cuda"


def _close(got, want, rtol=1e-4):
    scale = want.abs().max().clamp(min=1e-6)
    err = (got.float() - want.float()).abs().max()
    assert err <= rtol * scale, f"max err {err:.3e} vs scale {scale:.3e}"


def _segment_forward(q, k, v, bias, vcls, src, cls, qid, n_q):
    """Typed segment attention as index ops (cell_latents.py:546-567 form)."""
    heads, hd = q.shape[1], q.shape[2]
    score = (q[qid] * k[src]).sum(-1) / hd ** 0.5 + bias.t()[cls]
    mx = torch.full((n_q, heads), -1e30, device=q.device).index_reduce(0, qid, score.detach(), "amax")
    w = (score - mx[qid]).exp()
    den = torch.zeros(n_q, heads, device=q.device).index_add(0, qid, w)
    alpha = w / den[qid]
    val = v[src] + (vcls.view(-1, heads, hd)[cls] if vcls is not None else 0)
    return torch.zeros(n_q, heads, hd, device=q.device).index_add(0, qid, alpha[..., None] * val)


@pytest.mark.parametrize("heads,hd", [(8, 32), (4, 32), (2, 16)])
@pytest.mark.parametrize("with_vcls", [True, False])
def test_segment_attention_backward(heads, hd, with_vcls):
    g = torch.Generator().manual_seed(heads * 10 + hd)
    n_q, n_src, n_cls = 300, 120, 37
    runs = torch.randint(0, 12, (n_q,), generator=g)
    runs[5] = 0
    qid = torch.repeat_interleave(torch.arange(n_q), runs)
    src = torch.randint(0, n_src, (qid.numel(),), generator=g)
    cls = torch.randint(0, n_cls, (qid.numel(),), generator=g)
    seg_ptr = torch.cat([torch.zeros(1, dtype=torch.long), runs.cumsum(0)])
    t = [torch.randn(*s, generator=g) for s in ((n_q, heads, hd), (n_src, heads, hd), (n_src, heads, hd))]
    bias = torch.randn(heads, n_cls, generator=g)
    vcls = torch.randn(n_cls, heads * hd, generator=g) if with_vcls else None
    go = torch.randn(n_q, heads, hd, generator=g)
    dev = [x.to(DEV) for x in (seg_ptr, src, cls, qid)]
    q, k, v = (x.to(DEV).requires_grad_() for x in t)
    b = bias.to(DEV).requires_grad_()
    vc = vcls.to(DEV).requires_grad_() if with_vcls else None
    out = _segment_forward(q, k, v, b, vc, dev[1], dev[2], dev[3], n_q)
    out.backward(go.to(DEV))
    fwd, m, l = ops.segment_attention(q.detach().reshape(n_q, -1), k.detach().reshape(n_src, -1),
                                      v.detach().reshape(n_src, -1), b.detach(),
                                      vc.detach() if with_vcls else None, dev[0], dev[1], dev[2], stats=True)
    _close(fwd.view(n_q, heads, hd), out.detach())
    got = ops.segment_attention_backward(q.detach(), k.detach(), v.detach(), b.detach(),
                                         vc.detach() if with_vcls else None, dev[0], dev[1], dev[2], m, l,
                                         go.to(DEV))
    again = ops.segment_attention_backward(q.detach(), k.detach(), v.detach(), b.detach(),
                                           vc.detach() if with_vcls else None, dev[0], dev[1], dev[2], m, l,
                                           go.to(DEV))
    want = (q.grad, k.grad, v.grad, b.grad, vc.grad if with_vcls else None)
    for a, w, r in zip(got, want, again):
        if w is None:
            assert a is None
            continue
        _close(a, w)
        assert torch.equal(a, r), "backward is not deterministic"
    mb._lib.check_device_error()


@pytest.mark.parametrize("d", [16, 32, 64])
def test_stone_attention_backward(d):
    g = torch.Generator().manual_seed(d)
    p, heads, t = 5, 4, 150
    base = torch.randn(3, p, t, heads, d, generator=g)
    seq = torch.tensor([150, 1, 77, 64, 4], dtype=torch.int32)
    go = torch.randn(p, heads, t, d, generator=g)
    q, k, v = (base[i].to(DEV).transpose(1, 2).requires_grad_() for i in range(3))
    mask = torch.arange(t)[None, :] < seq[:, None].long()
    mk = mask.to(DEV)
    s = q @ k.transpose(-1, -2) / d ** 0.5
    s = s.masked_fill(~mk[:, None, None, :], float("-inf"))
    o = torch.softmax(s, -1) @ v
    o = o * mk[:, None, :, None]
    o.backward(go.to(DEV))
    out, lse = ops.fused_attention(q.detach(), k.detach(), v.detach(), seq.to(DEV), with_lse=True)
    _close(out, o.detach())
    got = ops.stone_attention_backward(q.detach(), k.detach(), v.detach(), seq.to(DEV), out, lse, go.to(DEV))
    again = ops.stone_attention_backward(q.detach(), k.detach(), v.detach(), seq.to(DEV), out, lse, go.to(DEV))
    for a, w, r in zip(got, (q.grad, k.grad, v.grad), again):
        _close(a, w, 2e-4)
        assert torch.equal(a, r)
    mb._lib.check_device_error()


def test_window_latent_backward():
    g = torch.Generator().manual_seed(3)
    p, heads, hd = 6, 8, 32
    pos = torch.sort(torch.randint(0, p, (400,), generator=g)).values
    pos[pos == 2] = 3  # a position without windows
    n_w = pos.numel()
    pd = pos.to(DEV)
    offsets, order = ops.window_latent_layout(pd, p)
    # read
    rq, rk, rv = (torch.randn(*s, generator=g).to(DEV).requires_grad_()
                  for s in ((p, 4, heads, hd), (n_w, heads, hd), (n_w, heads, hd)))
    go = torch.randn(p, 4, heads, hd, generator=g).to(DEV)
    s = torch.einsum("pqhd,whd->pqhw", rq, rk) / hd ** 0.5
    s = s.masked_fill((pd[None, :] != torch.arange(p, device=DEV)[:, None])[:, None, None, :], float("-inf"))
    a = torch.nan_to_num(torch.softmax(s, -1))
    ro = torch.einsum("pqhw,whd->pqhd", a, rv)
    ro.backward(go)
    out, m, l = ops.latent_read(rq.detach().reshape(p * 4, -1), rk.detach().reshape(n_w, -1),
                                rv.detach().reshape(n_w, -1), heads, offsets, order, stats=True)
    _close(out.view(ro.shape), ro.detach())
    got = ops.window_latent_read_backward(rq.detach(), rk.detach(), rv.detach(), offsets, order, pd, out, m, l, go)
    for x, w in zip(got, (rq.grad, rk.grad, rv.grad)):
        _close(x, w)
    # broadcast
    bq, bk, bv = (torch.randn(*s, generator=g).to(DEV).requires_grad_()
                  for s in ((n_w, heads, hd), (p, 4, heads, hd), (p, 4, heads, hd)))
    go = torch.randn(n_w, heads, hd, generator=g).to(DEV)
    s = torch.einsum("whd,wjhd->whj", bq, bk[pd]) / hd ** 0.5
    bo = torch.einsum("whj,wjhd->whd", torch.softmax(s, -1), bv[pd])
    bo.backward(go)
    out, m, l = ops.latent_broadcast(bq.detach().reshape(n_w, -1), bk.detach().reshape(p * 4, -1),
                                     bv.detach().reshape(p * 4, -1), heads, pd, p, stats=True)
    _close(out.view(bo.shape), bo.detach())
    got = ops.window_latent_broadcast_backward(bq.detach(), bk.detach(), bv.detach(), offsets, order, pd, m, l, go)
    for x, w in zip(got, (bq.grad, bk.grad, bv.grad)):
        _close(x, w)
    mb._lib.check_device_error()


@pytest.mark.parametrize("h", [32, 128, 256])
def test_encode_rows_backward(h):
    g = torch.Generator().manual_seed(h)
    n_pre, n_table, n_cells, e = 90, 31, 70, 600
    cell = torch.sort(torch.randint(0, n_cells, (e,), generator=g)).values
    win = torch.randint(0, n_pre, (e,), generator=g)
    cls = torch.randint(0, n_table, (e,), generator=g)
    pre = torch.randn(n_pre, h, generator=g).to(DEV).requires_grad_()
    table = torch.randn(n_table, h, generator=g).to(DEV).requires_grad_()
    go = torch.randn(n_cells, h, generator=g).to(DEV)
    d = [x.to(DEV) for x in (win, cls, cell)]
    out = torch.zeros(n_cells, h, device=DEV).index_add(0, d[2], torch.relu(pre[d[0]] + table[d[1]]))
    out.backward(go)
    fwd = ops.encode_rows(pre.detach(), table.detach(), d[0], d[1], d[2], torch.zeros_like(d[0]), n_cells)
    _close(fwd, out.detach())
    gp, gt = ops.encode_rows_backward(pre.detach(), table.detach(), d[0], d[1], d[2], go)
    _close(gp, pre.grad)
    _close(gt, table.grad)
    mb._lib.check_device_error()


def test_plugin_autograd_through_defined_ops():
    """torch.autograd through the plug-in's own ops (define()) matches the
    kernels' direct backward."""
    torch_ops = __import__("importlib").import_module("hexo-shrimp-bot_b200.torch_ops")
    torch_ops.define()
    g = torch.Generator().manual_seed(11)
    p, heads, t, d = 3, 4, 60, 32
    q, k, v = (torch.randn(p, heads, t, d, generator=g).to(DEV).requires_grad_() for _ in range(3))
    seq = torch.tensor([60, 7, 33], dtype=torch.int32, device=DEV)
    out, lse = torch.ops.mantis_b200.fused_attention(q, k, v, seq)
    go = torch.randn_like(out)
    out.backward(go)
    assert lse.numel() == 0  # fp32: the op keeps no log-sum-exp (reference contract); the backward recomputes it
    _, lse = ops.fused_attention(q.detach(), k.detach(), v.detach(), seq, with_lse=True)
    want = ops.stone_attention_backward(q.detach(), k.detach(), v.detach(), seq, out.detach(), lse, go)
    for a, w in zip((q.grad, k.grad, v.grad), want):
        assert torch.equal(a, w)
