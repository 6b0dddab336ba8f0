"""Op-level parity of the CUDA kernels (through the C ABI) against the CPU
oracle, on seeded inputs and the reference's op fixtures (tests/golden/ops.npz).

Tolerances: fp32 inputs 1e-5 abs / 1e-5 rel (fp32 math, different summation
order); bf16 inputs are compared against the oracle run on the same
bf16-rounded values, so the only differences are fp32 accumulation order:
2e-5 abs. Integer tables are bit-exact.
"""

from __future__ import annotations

import pytest
import torch

import golden_io
from golden_io import mb
from oracle import forward as O

pytestmark = pytest.mark.gpu
ops = mb.ops
DEV = "cuda"


def _fx():
    d = golden_io.load("ops.npz")
    return {k: torch.from_numpy(d[k]) for k in d.files}


def test_fused_attention_matches_reference_fixture():
    t = _fx()
    q, k, v, seq = (t[x].to(DEV) for x in ("att.q", "att.k", "att.v", "att.seq_lens"))
    out = ops.fused_attention(q, k, v, seq)
    torch.testing.assert_close(out.cpu(), t["att.out"], rtol=1e-5, atol=1e-5)
    # pad query rows are exactly zero (reference test_attention_kernel.py:202-228)
    assert torch.count_nonzero(out[2, :, 4:]) == 0


@pytest.mark.parametrize("d", [16, 32, 64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fused_attention_strided_ragged(d, dtype):
    """(P, T, A, D) storage viewed as (P, A, T, D), ragged seq_lens — the
    model's call pattern (model.py:633-640) on the reference's shape grid."""
    g = torch.Generator().manual_seed(d)
    for p, t in ((1, 2), (3, 65), (5, 200)):
        base = torch.randn(3, p, t, 2, d, generator=g).to(dtype)
        q, k, v = (base[i].to(DEV).transpose(1, 2) for i in range(3))
        seq = torch.randint(1, t + 1, (p,), generator=g, dtype=torch.int32)
        seq[0] = t
        out = ops.fused_attention(q, k, v, seq.to(DEV))
        assert out.stride() == q.stride()
        want = O.stone_attention(q.float().cpu(), k.float().cpu(), v.float().cpu(), seq.long())
        torch.testing.assert_close(out.float().cpu(), want, rtol=2e-2 if dtype == torch.bfloat16 else 1e-5,
                                   atol=2e-2 if dtype == torch.bfloat16 else 1e-5)


def test_segment_attention_matches_reference_fixture():
    t = _fx()
    qid, src, cls = t["seg.qid"], t["seg.src"], t["seg.cls"]
    n_q = t["seg.q"].shape[0]
    seg_ptr = torch.searchsorted(qid, torch.arange(n_q + 1))
    args = [x.to(DEV) for x in (t["seg.q"], t["seg.k"], t["seg.v"], t["seg.bias"])]
    out = ops.segment_attention(*args, t["seg.vcls"].to(DEV), seg_ptr.to(DEV), src.to(DEV), cls.to(DEV))
    torch.testing.assert_close(out.view(n_q, -1, t["seg.q"].shape[2]).cpu(), t["seg.out"], rtol=1e-5, atol=1e-5)
    plain = ops.segment_attention(*args, None, seg_ptr.to(DEV), src.to(DEV), cls.to(DEV))
    torch.testing.assert_close(plain.view(n_q, -1, t["seg.q"].shape[2]).cpu(), t["seg.out_plain"], rtol=1e-5,
                               atol=1e-5)
    assert torch.count_nonzero(out[2]) == 0


@pytest.mark.parametrize("heads,hd", [(2, 16), (4, 32), (8, 32), (2, 32)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_segment_attention_random_runs(heads, hd, dtype):
    g = torch.Generator().manual_seed(heads * 100 + hd)
    n_q, n_src, n_cls = 300, 90, 37
    runs = torch.randint(0, 19, (n_q,), generator=g)
    runs[::7] = 0  # empty runs
    qid = torch.repeat_interleave(torch.arange(n_q), runs)
    e = qid.numel()
    src = torch.randint(0, n_src, (e,), generator=g)
    cls = torch.randint(0, n_cls, (e,), generator=g)
    q = torch.randn(n_q, heads, hd, generator=g).to(dtype)
    k = torch.randn(n_src, heads, hd, generator=g).to(dtype)
    v = torch.randn(n_src, heads, hd, generator=g).to(dtype)
    bias = torch.randn(heads, n_cls, generator=g)
    vcls = torch.randn(n_cls, heads * hd, generator=g)
    seg_ptr = torch.cat([torch.zeros(1, dtype=torch.long), runs.cumsum(0)])
    out, m, l = ops.segment_attention(q.to(DEV), k.to(DEV), v.to(DEV), bias.to(DEV), vcls.to(DEV), seg_ptr.to(DEV),
                                      src.to(DEV), cls.to(DEV), stats=True)
    want = O.segment_attention(q.float(), k.float(), v.float(), bias, vcls, src, cls, qid)
    torch.testing.assert_close(out.view(n_q, heads, hd).cpu(), want, rtol=1e-5, atol=2e-5)
    empty = runs == 0
    assert torch.all(l.cpu()[empty] == 0) and torch.all(torch.isinf(m.cpu()[empty]))
    # skip_ptr: rows whose skip run is non-empty read zero
    skip = torch.cat([torch.zeros(1, dtype=torch.long), (torch.arange(n_q) % 3 == 0).long().cumsum(0)])
    out2 = ops.segment_attention(q.to(DEV), k.to(DEV), v.to(DEV), bias.to(DEV), vcls.to(DEV), seg_ptr.to(DEV),
                                 src.to(DEV), cls.to(DEV), skip_ptr=skip.to(DEV))
    masked = (torch.arange(n_q) % 3 == 0)
    assert torch.count_nonzero(out2.cpu()[masked]) == 0
    torch.testing.assert_close(out2.cpu()[~masked], out.cpu()[~masked])


def test_segment_attention_bad_index_is_reported_not_faulted():
    q = torch.randn(2, 1, 32, device=DEV)
    k = torch.randn(3, 1, 32, device=DEV)
    bias = torch.zeros(1, 4, device=DEV)
    seg_ptr = torch.tensor([0, 2, 3], device=DEV)
    src = torch.tensor([0, 7, 1], device=DEV)  # 7 is out of range
    cls = torch.tensor([0, 1, 2], device=DEV)
    mb._lib.check_device_error()  # clear
    ops.segment_attention(q, k, k, bias, None, seg_ptr, src, cls)
    with pytest.raises(ValueError, match="out of range"):
        mb._lib.check_device_error()
    mb._lib.check_device_error()  # cleared


def _grouped_case(heads, hd, seed, big=400):
    """Block-diagonal edges: group g's rows name only group g's sources
    (empty groups, empty runs and one group larger than a small stage)."""
    g = torch.Generator().manual_seed(seed)
    n_src_g = [5, 0, 37, big, 1, 60, 12]
    n_q_g = [40, 9, 0, 130, 7, 55, 33]
    q_off = torch.tensor([0] + n_q_g).cumsum(0)
    s_off = torch.tensor([0] + n_src_g).cumsum(0)
    runs, src = [], []
    for gi, (nq, ns) in enumerate(zip(n_q_g, n_src_g)):
        r = torch.randint(0, 25, (nq,), generator=g) if ns else torch.zeros(nq, dtype=torch.long)
        runs.append(r)
        src.append(s_off[gi] + torch.randint(0, max(ns, 1), (int(r.sum()),), generator=g))
    runs, src = torch.cat(runs), torch.cat(src)
    n_q, n_src, n_cls = int(q_off[-1]), int(s_off[-1]), 192
    cls = torch.randint(0, n_cls, (src.numel(),), generator=g)
    seg_ptr = torch.cat([torch.zeros(1, dtype=torch.long), runs.cumsum(0)])
    kv = torch.randn(n_src, 2 * heads * hd, generator=g).to(torch.bfloat16)
    q = torch.randn(n_q, heads * hd, generator=g).to(torch.bfloat16)
    bias = torch.randn(heads, n_cls, generator=g)
    vcls = torch.randn(n_cls, heads * hd, generator=g)
    return q, kv, bias, vcls, seg_ptr, src, cls, q_off, s_off, runs


@pytest.mark.parametrize("heads,hd", [(8, 32), (4, 16), (2, 32), (4, 64), (8, 8)])
@pytest.mark.parametrize("vdt", [None, torch.float32, torch.bfloat16])
@pytest.mark.parametrize("odt", [torch.float32, torch.bfloat16])
def test_segment_attention_grouped_matches_generic(heads, hd, vdt, odt):
    q, kv, bias, vcls, seg_ptr, src, cls, q_off, s_off, runs = (
        x.to(DEV) for x in _grouped_case(heads, hd, heads * 1000 + hd))
    h = heads * hd
    vc = None if vdt is None else vcls.to(vdt)

    def same(got, want, msg=""):
        # The grouped kernel rescales its softmax state once per chunk of
        # edges, the generic one once per edge: equal up to float rounding
        # (bf16 outputs: one bf16 step).
        if odt == torch.float32:
            torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5, msg=msg)
        else:
            torch.testing.assert_close(got.float(), want.float(), rtol=8e-3, atol=8e-3, msg=msg)

    want = ops.segment_attention(q, kv[:, :h], kv[:, h:], bias, vc, seg_ptr, src, cls, out_dtype=odt)
    for stage in (1024, 64, 1):  # all staged; the 400-source group from global memory; every group from global
        got = ops.segment_attention_grouped(q, kv[:, :h], kv[:, h:], bias, vc, seg_ptr, src, cls, q_off, s_off,
                                            stage, out_dtype=odt)
        torch.cuda.synchronize()
        same(got, want, f"stage_rows={stage}")
    skip = torch.cat([torch.zeros(1, dtype=torch.long, device=DEV),
                      (torch.arange(q.shape[0], device=DEV) % 3 == 0).long().cumsum(0)])
    want = ops.segment_attention(q, kv[:, :h], kv[:, h:], bias, vc, seg_ptr, src, cls, skip_ptr=skip, out_dtype=odt)
    got = ops.segment_attention_grouped(q, kv[:, :h], kv[:, h:], bias, vc, seg_ptr, src, cls, q_off, s_off, 1024,
                                        skip_ptr=skip, out_dtype=odt)
    same(got, want, "skip")
    mb._lib.check_device_error()


def test_segment_attention_grouped_against_oracle():
    q, kv, bias, vcls, seg_ptr, src, cls, q_off, s_off, runs = _grouped_case(8, 32, 7)
    qid = torch.repeat_interleave(torch.arange(q.shape[0]), runs)
    got = ops.segment_attention_grouped(q.to(DEV), kv[:, :256].to(DEV), kv[:, 256:].to(DEV), bias.to(DEV),
                                        vcls.to(DEV), seg_ptr.to(DEV), src.to(DEV), cls.to(DEV), q_off.to(DEV),
                                        s_off.to(DEV), 1024, out_dtype=torch.float32)
    want = O.segment_attention(q.float().view(-1, 8, 32), kv[:, :256].float().view(-1, 8, 32),
                               kv[:, 256:].float().view(-1, 8, 32), bias, vcls, src, cls, qid)
    torch.testing.assert_close(got.view(-1, 8, 32).cpu(), want, rtol=1e-5, atol=2e-5)


def test_segment_attention_grouped_cross_group_edge_is_reported():
    q, kv, bias, vcls, seg_ptr, src, cls, q_off, s_off, runs = _grouped_case(8, 32, 3)
    src = src.clone()
    src[0] = int(s_off[3])  # a row of group 0 naming a source of group 3
    mb._lib.check_device_error()  # clear
    ops.segment_attention_grouped(q.to(DEV), kv[:, :256].to(DEV), kv[:, 256:].to(DEV), bias.to(DEV), None,
                                  seg_ptr.to(DEV), src.to(DEV), cls.to(DEV), q_off.to(DEV), s_off.to(DEV), 1024)
    with pytest.raises(ValueError, match="out of range"):
        mb._lib.check_device_error()
    mb._lib.check_device_error()  # cleared


def test_window_latents_match_reference_fixture():
    t = _fx()
    pos = t["win.pos"].to(DEV)
    offsets, order = ops.window_latent_layout(pos, 4)
    rd = ops.read_attention(t["win.rq"].to(DEV), t["win.rk"].to(DEV), t["win.rv"].to(DEV), pos, offsets, order)
    torch.testing.assert_close(rd.cpu(), t["win.read"], rtol=1e-5, atol=1e-5)
    assert torch.count_nonzero(rd[1]) == 0
    bc = ops.broadcast_attention(t["win.bq"].to(DEV), t["win.bk"].to(DEV), t["win.bv"].to(DEV), pos, offsets, order)
    torch.testing.assert_close(bc.cpu(), t["win.bcast"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("heads,hd", [(4, 32), (8, 32), (2, 16)])
def test_window_latents_random(heads, hd):
    g = torch.Generator().manual_seed(hd + heads)
    p = 7
    counts = torch.tensor([0, 1, 40, 300, 5, 1000, 33])
    pos = torch.repeat_interleave(torch.arange(p), counts)
    nw = pos.numel()
    q = torch.randn(p, 4, heads, hd, generator=g)
    k = torch.randn(nw, heads, hd, generator=g)
    v = torch.randn(nw, heads, hd, generator=g)
    offsets, order = ops.window_latent_layout(pos.to(DEV), p)
    rd = ops.read_attention(q.to(DEV), k.to(DEV), v.to(DEV), pos.to(DEV), offsets, order)
    torch.testing.assert_close(rd.cpu(), O.window_read(q, k, v, pos), rtol=1e-5, atol=2e-5)
    bq = torch.randn(nw, heads, hd, generator=g)
    bc = ops.broadcast_attention(bq.to(DEV), q.to(DEV), k[:p * 4].reshape(p, 4, heads, hd).to(DEV), pos.to(DEV),
                                 offsets, order)
    torch.testing.assert_close(bc.cpu(), O.window_broadcast(bq, q, k[:p * 4].reshape(p, 4, heads, hd), pos),
                               rtol=1e-5, atol=2e-5)


def test_row_encoder_matches_reference_fixture():
    t = _fx()
    out = ops.encode_rows(*(t[x].to(DEV) for x in ("row.pre", "row.table", "row.win", "row.cls", "row.cell")),
                          t["row.cell"].to(DEV), 5)
    torch.testing.assert_close(out.cpu(), t["row.out"], rtol=1e-5, atol=1e-5)


def test_run_reductions_against_oracle():
    g = torch.Generator().manual_seed(3)
    n_src, n_dest, h = 50, 40, 256
    runs = torch.randint(0, 7, (n_dest,), generator=g)
    dest = torch.repeat_interleave(torch.arange(n_dest), runs)
    gather = torch.randint(0, n_src, (dest.numel(),), generator=g)
    vals = torch.randn(n_src, h, generator=g)
    for dtype in (torch.float32, torch.bfloat16):
        x = vals.to(dtype)
        want = O.row_sum(x.float(), gather, dest, n_dest)
        got = ops.class_row_sum(x.to(DEV), gather.to(DEV), dest.to(DEV), n_dest)
        torch.testing.assert_close(got.cpu(), want, rtol=1e-5, atol=1e-5)
        got = ops.aggregate_to_windows(x.to(DEV), gather.to(DEV), dest.to(DEV), dest.to(DEV), gather.to(DEV), n_dest)
        assert got.dtype == dtype
        torch.testing.assert_close(got.float().cpu(), want.to(dtype).float(), rtol=1e-2, atol=1e-2)


def test_cell_pass_against_oracle():
    cfg, P, batch, _, _ = golden_io.forward_case("default")
    g = torch.Generator().manual_seed(4)
    x = torch.randn(batch.n_windows, 32, generator=g)
    emb = torch.randn(726, 32, generator=g)
    b = batch.to(DEV)
    got = ops.cell_pass(x.to(DEV), emb.to(DEV), b.relay_cell_ptr, b.relay_window, b.relay_class, b.relay_win_ptr,
                        b.relay_wcell, b.relay_cls_ptr, b.relay_ccell)
    want = O.cell_pass(x, emb, batch.dec_cell, batch.dec_window, batch.dec_class)
    torch.testing.assert_close(got.cpu(), want, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("name", ["cellnodes", "full", "uncovered"])
def test_integer_tables_bit_exact(name):
    """Device CSR derivations equal the reference's torch compositions."""
    cfg, P, batch, _, _ = golden_io.forward_case(name)
    b = batch.to(DEV)
    n_w, n_c, n_s = batch.n_windows, batch.n_cells, batch.n_stones
    for n_cells in (n_c, -1):
        got = ops.cell_tables(b.dec_cell, b.dec_window, b.dec_class, n_w, 726, n_cells)
        want = O.cell_tables(batch.dec_cell, batch.dec_window, batch.dec_class, n_w, n_cells)
        for k in ("covered", "cell_ptr", "edge_window", "edge_class", "edge_cell", "win_ptr", "edge_wcell",
                  "edge_wclass", "edge_wwin"):
            assert torch.equal(getattr(got, k).cpu(), want[k]), k
    cov = O.cell_tables(batch.dec_cell, batch.dec_window, batch.dec_class, n_w, n_c)["covered"]
    rcls = batch.radius_orbit + 48 * (batch.radius_own + 2 * batch.radius_on_axis)
    for scope in (False, True):
        got = ops.edge_tables(b.radius_src, b.radius_dst, rcls.to(DEV), cov.to(DEV), n_s, n_c, 192, scope)
        want = O.edge_tables(batch.radius_src, batch.radius_dst, rcls, cov, n_s, n_c, scope)
        pairs = dict(cell_ptr="dst_ptr", edge_window="edge_src", edge_class="edge_class", edge_cell="edge_dst",
                     win_ptr="src_ptr", edge_wcell="edge_sdst", edge_wclass="edge_sclass", edge_wwin="edge_ssrc")
        for k, kw in pairs.items():
            assert torch.equal(getattr(got, k).cpu(), want[kw]), (scope, k)
    plan = ops.incidence_plan(b.inc_stone, b.inc_window, b.inc_class)
    want = O.incidence_plan(batch.inc_stone, batch.inc_window, batch.inc_class)
    for a_, b_ in zip(plan, want):
        assert torch.equal(a_.cpu(), b_)
    pos = batch.window_slot // batch.value_valid.shape[1]
    off, order = ops.window_latent_layout(pos.to(DEV), batch.n_pos)
    woff, worder = O.window_latent_layout(pos, batch.n_pos)
    assert torch.equal(off.cpu(), woff) and torch.equal(order.cpu(), worder)


def test_layer_norm_and_compose():
    g = torch.Generator().manual_seed(9)
    x = torch.randn(333, 256, generator=g) * 3 + 1
    gam, bet = torch.randn(256, generator=g), torch.randn(256, generator=g)
    got = ops.layer_norm(x.to(DEV), gam.to(DEV), bet.to(DEV), out_dtype=torch.float32)
    torch.testing.assert_close(got.cpu(), torch.nn.functional.layer_norm(x, (256,), gam, bet), rtol=1e-5, atol=1e-5)
    critic = torch.randn(100, 3, generator=g) * 2
    offs = torch.tensor([0, 1, 40, 100])
    qs, qv = ops.compose(critic.to(DEV), offs.to(DEV), 0.2)
    torch.testing.assert_close(qv.cpu(), O.compose_q(critic), rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(qs.cpu(), O.compose_acting_q(critic, offs, 0.2), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_native_linear(dtype):
    g = torch.Generator().manual_seed(1)
    a = torch.randn(1000, 96, generator=g).to(dtype)
    w = torch.randn(80, 96, generator=g).to(dtype)
    b = torch.randn(80, generator=g)
    got = ops.linear_native(a.to(DEV), w.to(DEV), b.to(DEV), relu=True, out_dtype=torch.float32)
    want = torch.relu(a.float() @ w.float().t() + b)
    torch.testing.assert_close(got.cpu(), want, rtol=1e-4, atol=1e-4)


# ------------------------------------------------ radius read on packed edges
def _degree_order(seg_ptr, q_off):
    """Each group's rows by ascending run length (the engine's order)."""
    runs = seg_ptr[1:] - seg_ptr[:-1]
    grp = torch.repeat_interleave(torch.arange(q_off.numel() - 1, device=seg_ptr.device), q_off[1:] - q_off[:-1])
    return torch.argsort(grp * 4096 + runs, stable=True)


@pytest.mark.parametrize("heads", [8, 2])
@pytest.mark.parametrize("vdt", [None, torch.bfloat16])
@pytest.mark.parametrize("odt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("ordered", [False, True])
@pytest.mark.parametrize("slotted", [False, True])
def test_radius_read_matches_generic(heads, vdt, odt, ordered, slotted):
    q, kv, bias, vcls, seg_ptr, src, cls, q_off, s_off, runs = (
        x.to(DEV) for x in _grouped_case(heads, 32, heads * 77 + 5))
    h = heads * 32
    vc = None if vdt is None else vcls.to(vdt)
    packed = ops.radius_pack(src, cls, seg_ptr, q_off, s_off, kv.shape[0], bias.shape[1])
    order = _degree_order(seg_ptr, q_off) if ordered else None
    want = ops.segment_attention(q, kv[:, :h], kv[:, h:], bias, vc, seg_ptr, src, cls, out_dtype=torch.float32)
    slots, pk = ops.radius_slots(packed, seg_ptr, q_off, order) if slotted else (None, packed)
    for stage in (1024, 64, 1):  # all staged; the 400-source group from global memory; every group from global
        got = ops.radius_read(q, kv[:, :h], kv[:, h:], bias, vc, seg_ptr, pk, q_off, s_off, stage, order=order,
                              out_dtype=odt, slots=slots)
        torch.cuda.synchronize()
        tol = 1e-5 if odt == torch.float32 else 8e-3
        torch.testing.assert_close(got.float(), want, rtol=tol, atol=tol, msg=f"stage_rows={stage}")
    skip = torch.cat([torch.zeros(1, dtype=torch.long, device=DEV),
                      (torch.arange(q.shape[0], device=DEV) % 3 == 0).long().cumsum(0)])
    want = ops.segment_attention(q, kv[:, :h], kv[:, h:], bias, vc, seg_ptr, src, cls, skip_ptr=skip,
                                 out_dtype=torch.float32)
    slots, pk = ops.radius_slots(packed, seg_ptr, q_off, order, skip) if slotted else (None, packed)
    got = ops.radius_read(q, kv[:, :h], kv[:, h:], bias, vc, seg_ptr, pk, q_off, s_off, 1024, order=order,
                          skip_ptr=skip, out_dtype=odt, slots=slots)
    tol = 1e-5 if odt == torch.float32 else 8e-3
    torch.testing.assert_close(got.float(), want, rtol=tol, atol=tol, msg="skip")
    mb._lib.check_device_error()


def test_radius_read_against_oracle_and_bad_edge():
    q, kv, bias, vcls, seg_ptr, src, cls, q_off, s_off, runs = _grouped_case(8, 32, 11)
    qid = torch.repeat_interleave(torch.arange(q.shape[0]), runs)
    d = [x.to(DEV) for x in (q, kv, bias, vcls, seg_ptr, src, cls, q_off, s_off)]
    packed = ops.radius_pack(d[5], d[6], d[4], d[7], d[8], kv.shape[0], 192)
    got = ops.radius_read(d[0], d[1][:, :256], d[1][:, 256:], d[2], d[3].to(torch.bfloat16), d[4], packed, d[7],
                          d[8], 1024, order=_degree_order(d[4], d[7]), out_dtype=torch.float32)
    want = O.segment_attention(q.float().view(-1, 8, 32), kv[:, :256].float().view(-1, 8, 32),
                               kv[:, 256:].float().view(-1, 8, 32), bias, vcls.to(torch.bfloat16).float(), src, cls,
                               qid)
    torch.testing.assert_close(got.view(-1, 8, 32).cpu(), want, rtol=1e-5, atol=2e-5)
    mb._lib.check_device_error()
    bad = d[5].clone()
    bad[0] = int(s_off[3])  # a row of group 0 naming a stone of group 3: refused when packing
    packed = ops.radius_pack(bad, d[6], d[4], d[7], d[8], kv.shape[0], 192)
    assert int(packed[0]) == -1
    with pytest.raises(ValueError, match="out of range"):
        mb._lib.check_device_error()
    mb._lib.check_device_error()  # cleared


# ------------------------------------------------ stone attention on tcgen05
def _ragged_tokens(lengths, heads, seed):
    g = torch.Generator().manual_seed(seed)
    tok_off = torch.tensor([0] + list(lengths)).cumsum(0)
    qkv = (torch.randn(int(tok_off[-1]), 3 * heads * 32, generator=g) * 1.5).to(torch.bfloat16)
    return qkv, tok_off


def _ragged_oracle(qkv, tok_off, heads, max_queries=-1):
    h = heads * 32
    outs = []
    for p in range(tok_off.numel() - 1):
        a, b = int(tok_off[p]), int(tok_off[p + 1])
        x = qkv[a:b].float()
        q, k, v = (x[:, i * h:(i + 1) * h].view(b - a, heads, 32).transpose(0, 1) for i in range(3))
        o = torch.softmax(q @ k.transpose(1, 2) / 32 ** 0.5, -1) @ v
        o = o.transpose(0, 1).reshape(b - a, h)
        outs.append(o[:max_queries] if max_queries >= 0 else o)
    return torch.cat(outs)


@pytest.mark.parametrize("lengths", [[4, 5, 37, 128, 129, 200], [304, 4, 257, 320, 300], [64, 63, 65, 256]])
@pytest.mark.parametrize("engine", [1, 0])
def test_stone_attention_ragged_tensor_cores(lengths, engine):
    """[latents; stones] attention on the ragged token layout at the lengths
    of late positions (T up to 320 keys, past one 256-column MMA and two
    128-query tiles), on the tensor cores (engine 1) and on the CUDA cores
    (engine 0), against fp32 attention on the same bf16 rows; the latent-only
    read of the last block (max_queries = 4, compact output) too."""
    heads = 8
    qkv, tok_off = _ragged_tokens(lengths, heads, sum(lengths))
    mb._lib.call("mb_stone_attention_engine", engine)
    try:
        d = qkv.to(DEV)
        to = tok_off.to(DEV)
        got = ops.stone_attention_ragged(d, to, heads, max(lengths))
        lat = ops.stone_attention_ragged(d, to, heads, max(lengths), max_queries=4, out_dtype=torch.float32)
        torch.cuda.synchronize()
    finally:
        mb._lib.call("mb_stone_attention_engine", 1)
    want = _ragged_oracle(qkv, tok_off, heads)
    torch.testing.assert_close(got.float().cpu(), want, rtol=2e-2, atol=2e-2)
    want4 = _ragged_oracle(qkv, tok_off, heads, 4)
    torch.testing.assert_close(lat.cpu(), want4, rtol=1e-2, atol=1e-2)
    mb._lib.check_device_error()


def test_stone_attention_padded_tensor_cores_zero_pad_rows():
    """The padded (P, A, T, D) entry (mantisnet::fused_attention) on the
    tensor cores: rows past seq_lens read zero, a position with one key."""
    g = torch.Generator().manual_seed(9)
    p, t = 4, 300
    base = torch.randn(3, p, t, 8, 32, generator=g).to(torch.bfloat16)
    q, k, v = (base[i].to(DEV).transpose(1, 2) for i in range(3))
    seq = torch.tensor([300, 1, 129, 64], dtype=torch.int32)
    out = ops.fused_attention(q, k, v, seq.to(DEV))
    want = O.stone_attention(q.float().cpu(), k.float().cpu(), v.float().cpu(), seq.long())
    torch.testing.assert_close(out.float().cpu(), want, rtol=2e-2, atol=2e-2)
    assert torch.count_nonzero(out[1, :, 1:]) == 0 and torch.count_nonzero(out[2, :, 129:]) == 0
    mb._lib.check_device_error()
