"""Tensor-level wrappers over the C ABI.

Two layers:

1. Thin wrappers (``run_reduce``, ``segment_attention``, ...) used by the
   model: they take CUDA tensors (row-major, unit inner stride, views allowed)
   and launch on the current stream.
2. The reference's operator surface, same names, argument meaning and error
   classes (``ValueError`` for bad arguments): ``fused_attention``,
   ``aggregate_to_windows``, ``aggregate_to_stones``, ``class_row_sum``,
   ``incidence_row_sum``, ``cell_attention``, ``cell_attention_plain``,
   ``read_attention``/``broadcast_attention``, ``window_latent_layout``,
   ``encode_rows``, ``cell_pass``, ``cell_tables``, ``edge_tables``,
   ``incidence_plan`` (reference python/mantisnet/mantisnet/{attention,
   message_passing,cell_latents,cell_nodes,window_latents,row_encoder,
   relay}.py). There is no CPU path: a non-CUDA tensor raises.
"""

from __future__ import annotations

import ctypes
import math
from typing import NamedTuple

import torch

from . import _lib
from ._lib import call, dtype_code, ptr, stream_of

_I64 = torch.int64


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("the B200 kernels take CUDA tensors only (no CPU fallback)")


def _rowmajor(t, name):
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a row-major 2-D tensor with unit inner stride")


def _i64(t, name):
    if t.dtype != _I64:
        raise ValueError(f"{name} must have dtype int64")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _bits(n: int) -> int:
    return max(1, int(n - 1).bit_length()) if n > 1 else 1


# --------------------------------------------------------------- tables

def csr(keys: torch.Tensor, n_dest: int) -> torch.Tensor:
    """ptr[d] = searchsorted(keys, d, left) for d in [0, n_dest]."""
    _cuda(keys)
    _i64(keys, "keys")
    out = torch.empty(n_dest + 1, dtype=_I64, device=keys.device)
    call("mb_csr_from_sorted", ptr(keys), keys.numel(), n_dest, ptr(out), stream_of(keys.device))
    return out


def argsort(keys: torch.Tensor, bound: int):
    """Stable argsort of int64 keys in [0, bound): (sorted_keys, order)."""
    _cuda(keys)
    _i64(keys, "keys")
    n = keys.numel()
    sk = torch.empty_like(keys)
    order = torch.empty_like(keys)
    if n == 0:
        return sk, order
    bits = _bits(bound)
    need = ctypes.c_int64(0)
    call("mb_argsort_workspace", n, bits, ctypes.byref(need))
    ws = torch.empty(need.value, dtype=torch.uint8, device=keys.device)
    call("mb_argsort", ptr(keys), n, bits, ptr(sk), ptr(order), ptr(ws), need.value, stream_of(keys.device))
    return sk, order


def gather_i64(src: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    out = torch.empty(idx.shape[0], dtype=_I64, device=idx.device)
    call("mb_gather_i64", ptr(src), src.numel(), ptr(idx), idx.numel(), ptr(out), stream_of(idx.device))
    return out


def radius_class(orbit, own, on_axis, order=None) -> torch.Tensor:
    out = torch.empty(orbit.shape[0], dtype=_I64, device=orbit.device)
    call("mb_radius_class", ptr(orbit), ptr(own), ptr(on_axis), ptr(order), orbit.numel(), ptr(out),
         stream_of(orbit.device))
    return out


def div_i64(x: torch.Tensor, divisor: int) -> torch.Tensor:
    out = torch.empty_like(x)
    call("mb_div_i64", ptr(x), x.numel(), int(divisor), ptr(out), stream_of(x.device))
    return out


# ------------------------------------------------------- thin wrappers

def run_reduce(values, gather, ptr_, n_dest, add=None, add_idx=None, out=None, out_dtype=torch.float32):
    """out[d] = sum_{e in run d} values[gather[e]] (+ add[add_idx[d]]), fp32 accumulation."""
    _cuda(values, gather, ptr_)
    _rowmajor(values, "values")
    width = values.shape[1]
    if out is None:
        out = torch.empty(n_dest, width, dtype=out_dtype, device=values.device)
    n_add = 0
    if add is not None:
        _rowmajor(add, "add")
        n_add = add.shape[0]
    call("mb_run_reduce", ptr(values), dtype_code(values.dtype), values.stride(0), values.shape[0], ptr(gather),
         ptr(ptr_), n_dest, width, ptr(add), add.stride(0) if add is not None else 0, ptr(add_idx), n_add,
         ptr(out), dtype_code(out.dtype), out.stride(0), stream_of(values.device))
    return out


def row_encode(pre, table, edge_window, edge_class, cell_ptr, n_cells, empty_counts=None, empty_base=None,
               empty_cls=None, out_dtype=torch.float32, out=None):
    """Action-row encoder (K5); ``out`` may be a row-strided column view."""
    _cuda(pre, table, edge_window, edge_class, cell_ptr)
    h = pre.shape[1]
    if out is None:
        out = torch.empty(n_cells, h, dtype=out_dtype, device=pre.device)
    elif out.shape != (n_cells, h) or out.stride(1) != 1:
        raise ValueError("row_encode out must be (n_cells, h) with unit column stride")
    n_empty = empty_cls.numel() if empty_cls is not None else 0
    call("mb_row_encode", ptr(pre), dtype_code(pre.dtype), pre.shape[0], ptr(table), table.shape[0],
         ptr(edge_window), ptr(edge_class), ptr(cell_ptr), n_cells,
         ptr(empty_counts), ptr(empty_base), ptr(empty_cls), n_empty, h, ptr(out), dtype_code(out.dtype),
         out.stride(0), stream_of(pre.device))
    return out


def segment_attention(q, k, v, bias, vcls, seg_ptr, src, cls, skip_ptr=None, out=None, out_dtype=torch.float32,
                      stats=False):
    """Typed segment attention (K3). q (n_q, A, d) or (n_q, H) rows; k/v may
    be column views of one fused projection (same row stride)."""
    _cuda(q, k, v, bias, seg_ptr)
    heads = bias.shape[0]
    q2 = q.reshape(q.shape[0], -1) if q.dim() == 3 else q
    k2 = k.reshape(k.shape[0], -1) if k.dim() == 3 else k
    v2 = v.reshape(v.shape[0], -1) if v.dim() == 3 else v
    for t, n in ((q2, "q"), (k2, "k"), (v2, "v")):
        _rowmajor(t, n)
    if k2.stride(0) != v2.stride(0):
        raise ValueError("k and v must share a row stride")
    if not (q2.dtype == k2.dtype == v2.dtype):
        raise ValueError("q, k, and v must have one dtype")
    n_q, width = q2.shape
    hd = width // heads
    if out is None:
        out = torch.empty(n_q, width, dtype=out_dtype, device=q.device)
    m = l = None
    if stats:
        m = torch.empty(n_q, heads, dtype=torch.float32, device=q.device)
        l = torch.empty_like(m)
    bias32 = bias if (bias.dtype == torch.float32 and bias.is_contiguous()) else bias.float().contiguous()
    if vcls is not None and not (vcls.dtype in (torch.float32, torch.bfloat16) and vcls.is_contiguous()):
        vcls = vcls.float().contiguous()
    call("mb_segment_attention", ptr(q2), q2.stride(0), ptr(k2), ptr(v2), k2.stride(0), dtype_code(q2.dtype),
         n_q, k2.shape[0], heads, hd, ptr(bias32), bias32.shape[1], ptr(vcls),
         dtype_code(vcls.dtype) if vcls is not None else 0, ptr(seg_ptr), ptr(src), ptr(cls),
         ptr(skip_ptr), ptr(out), dtype_code(out.dtype), out.stride(0), ptr(m), ptr(l), stream_of(q.device))
    return (out, m, l) if stats else out


def segment_attention_grouped(q, k, v, bias, vcls, seg_ptr, src, cls, q_off, s_off, stage_rows, skip_ptr=None,
                              out=None, out_dtype=torch.bfloat16):
    """Segment attention over a block-diagonal edge set (the radius read:
    group g = position g, its cells [q_off[g], q_off[g+1]) attend only to its
    stones [s_off[g], s_off[g+1])). Same result as ``segment_attention`` up
    to float rounding; each group's K/V columns are staged in shared memory
    (up to ``stage_rows`` sources per group). bf16 q/k/v only."""
    _cuda(q, k, v, bias, seg_ptr, q_off, s_off)
    heads = bias.shape[0]
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _rowmajor(t, n)
    if k.stride(0) != v.stride(0):
        raise ValueError("k and v must share a row stride")
    if not (q.dtype == k.dtype == v.dtype == torch.bfloat16):
        raise ValueError("segment_attention_grouped needs bf16 q, k and v")
    n_q, width = q.shape
    if out is None:
        out = torch.empty(n_q, width, dtype=out_dtype, device=q.device)
    bias32 = bias if (bias.dtype == torch.float32 and bias.is_contiguous()) else bias.float().contiguous()
    if vcls is not None and not (vcls.dtype in (torch.float32, torch.bfloat16) and vcls.is_contiguous()):
        vcls = vcls.float().contiguous()
    call("mb_segment_attention_grouped", ptr(q), q.stride(0), ptr(k), ptr(v), k.stride(0), dtype_code(q.dtype),
         n_q, k.shape[0], heads, width // heads, ptr(bias32), bias32.shape[1], ptr(vcls),
         dtype_code(vcls.dtype) if vcls is not None else 0, ptr(seg_ptr), ptr(src), ptr(cls), ptr(skip_ptr),
         ptr(q_off), ptr(s_off), q_off.shape[0] - 1, max(int(stage_rows), 1), ptr(out), dtype_code(out.dtype),
         out.stride(0), stream_of(q.device))
    return out


def radius_pack(src, cls, seg_ptr, q_off, s_off, n_src: int, n_cls: int) -> torch.Tensor:
    """int32 packed radius edges (local stone << 11 | class) for
    ``radius_read``; computed once per forward, shared by every block."""
    _cuda(src, cls, seg_ptr, q_off, s_off)
    for t, n in ((src, "src"), (cls, "cls"), (seg_ptr, "seg_ptr"), (q_off, "q_off"), (s_off, "s_off")):
        _i64(t, n)
    packed = torch.empty(src.shape[0], dtype=torch.int32, device=src.device)
    call("mb_radius_pack_edges", ptr(src), ptr(cls), ptr(seg_ptr), ptr(q_off), ptr(s_off), q_off.shape[0] - 1,
         seg_ptr.shape[0] - 1, src.shape[0], n_src, n_cls, ptr(packed), stream_of(src.device))
    return packed


def radius_slots(packed, seg_ptr, q_off, order=None, skip_ptr=None):
    """(slots, packed_slots) for ``radius_read``: per slot of ``order``
    (ascending rows when None) the row, where its edges start in
    ``packed_slots`` and its edge count (0 for a row ``skip_ptr`` skips), and
    the packed edges (``radius_pack``) copied into slot order, each run padded
    to a multiple of four. Computed once per forward."""
    _cuda(packed, seg_ptr, q_off)
    _i64(seg_ptr, "seg_ptr")
    _i64(q_off, "q_off")
    for t, n in ((order, "order"), (skip_ptr, "skip_ptr")):
        if t is not None:
            _cuda(t)
            _i64(t, n)
    n_q, n_groups, n_edges = seg_ptr.shape[0] - 1, q_off.shape[0] - 1, packed.shape[0]
    length = ctypes.c_int64(0)
    call("mb_radius_slots_size", n_q, n_groups, n_edges, ctypes.byref(length))
    slots = torch.empty(n_q, 4, dtype=torch.int32, device=seg_ptr.device)
    packed_slots = torch.empty(length.value, dtype=torch.int32, device=seg_ptr.device)
    call("mb_radius_slots", ptr(packed), ptr(seg_ptr), ptr(skip_ptr), ptr(order), ptr(q_off), n_groups, n_q, n_edges,
         ptr(slots), ptr(packed_slots), length.value, stream_of(seg_ptr.device))
    return slots, packed_slots


def radius_read(q, k, v, bias, vcls, seg_ptr, packed, q_off, s_off, stage_rows, order=None, skip_ptr=None, out=None,
                out_dtype=torch.bfloat16, slots=None):
    """The radius read on packed edges: same result as
    ``segment_attention_grouped`` up to float rounding. head_dim 32, bf16
    q/k/v (and class value rows). With ``slots`` (the table of
    ``radius_slots``), ``packed`` must be its slot-ordered copy of the edges;
    ``order`` / ``seg_ptr`` / ``skip_ptr`` are then not read."""
    _cuda(q, k, v, bias, seg_ptr, packed, q_off, s_off)
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _rowmajor(t, n)
    if k.stride(0) != v.stride(0):
        raise ValueError("k and v must share a row stride")
    if not (q.dtype == k.dtype == v.dtype == torch.bfloat16):
        raise ValueError("radius_read needs bf16 q, k and v")
    if packed.dtype != torch.int32:
        raise ValueError("packed edges must be int32 (radius_pack)")
    if slots is not None and (slots.dtype != torch.int32 or slots.shape != (q.shape[0], 4) or not slots.is_contiguous()):
        raise ValueError("slots must be the (n_q, 4) int32 table of radius_slots")
    heads = bias.shape[0]
    n_q, width = q.shape
    if out is None:
        out = torch.empty(n_q, width, dtype=out_dtype, device=q.device)
    bias32 = bias if (bias.dtype == torch.float32 and bias.is_contiguous()) else bias.float().contiguous()
    if vcls is not None and not (vcls.dtype == torch.bfloat16 and vcls.is_contiguous()):
        vcls = vcls.to(torch.bfloat16).contiguous()
    call("mb_radius_read", ptr(q), q.stride(0), ptr(k), ptr(v), k.stride(0), n_q, k.shape[0], heads, width // heads,
         ptr(bias32), bias32.shape[1], ptr(vcls), ptr(seg_ptr), ptr(packed), ptr(skip_ptr), ptr(q_off), ptr(s_off),
         ptr(order), ptr(slots), q_off.shape[0] - 1, max(int(stage_rows), 1), ptr(out), dtype_code(out.dtype),
         out.stride(0), stream_of(q.device))
    return out


def radius_supported(heads: int, width: int, dtype) -> bool:
    """Whether ``radius_read`` takes this shape."""
    return dtype == torch.bfloat16 and width == heads * 32 and width % 64 == 0


def grouped_supported(heads: int, width: int, dtype) -> bool:
    """Whether ``segment_attention_grouped`` takes this shape."""
    hd = width // heads
    return dtype == torch.bfloat16 and width % 64 == 0 and hd % 8 == 0 and 64 % hd == 0


def stone_attention_ragged(qkv, tok_off, heads, max_tokens, max_queries=-1, out=None, out_dtype=None):
    """Attention over [latents; stones] per position on the token layout:
    qkv (N_tok, 3H) = [q | k | v]. With max_queries=4 the output is compact
    (P*4, H); otherwise (N_tok, H)."""
    _rowmajor(qkv, "qkv")
    h = qkv.shape[1] // 3
    hd = h // heads
    n_pos = tok_off.shape[0] - 1
    out_dtype = out_dtype or qkv.dtype
    compact = max_queries >= 0
    if out is None:
        rows = n_pos * max_queries if compact else qkv.shape[0]
        out = torch.empty(rows, h, dtype=out_dtype, device=qkv.device)
    es = qkv.element_size()
    call("mb_stone_attention", ptr(qkv), qkv.data_ptr() + h * es, qkv.data_ptr() + 2 * h * es,
         dtype_code(qkv.dtype), n_pos, heads, hd, 0, hd, qkv.stride(0), None, 0, ptr(tok_off), max_tokens,
         max_queries, ptr(out), dtype_code(out.dtype), max_queries * out.stride(0) if compact else 0, hd,
         out.stride(0), None, stream_of(qkv.device))
    return out


def latent_read(q, k, v, heads, offsets, order, out_dtype=torch.float32, stats=False):
    """q (P*4, H) rows, k/v (N_w, H) rows (views of a fused kv allowed)."""
    _rowmajor(q, "q"); _rowmajor(k, "k"); _rowmajor(v, "v")
    n_pos = offsets.shape[0] - 1
    h = q.shape[1]
    out = torch.empty(n_pos * 4, h, dtype=out_dtype, device=q.device)
    m = l = None
    if stats:
        m = torch.empty(n_pos * 4, heads, dtype=torch.float32, device=q.device)
        l = torch.empty_like(m)
    call("mb_window_latent_read", ptr(q), q.stride(0), ptr(k), ptr(v), k.stride(0), dtype_code(q.dtype), n_pos,
         k.shape[0], heads, h // heads, ptr(offsets), ptr(order), ptr(out), dtype_code(out_dtype), ptr(m), ptr(l),
         stream_of(q.device))
    return (out, m, l) if stats else out


def latent_broadcast(q, k, v, heads, window_pos, n_pos, out_dtype=torch.float32, stats=False):
    _rowmajor(q, "q"); _rowmajor(k, "k"); _rowmajor(v, "v")
    n_w, h = q.shape
    out = torch.empty(n_w, h, dtype=out_dtype, device=q.device)
    m = l = None
    if stats:
        m = torch.empty(n_w, heads, dtype=torch.float32, device=q.device)
        l = torch.empty_like(m)
    call("mb_window_latent_broadcast", ptr(q), q.stride(0), ptr(k), ptr(v), k.stride(0), dtype_code(q.dtype),
         n_pos, n_w, heads, h // heads, ptr(window_pos), ptr(out), dtype_code(out_dtype), ptr(m), ptr(l),
         stream_of(q.device))
    return (out, m, l) if stats else out


def latent_mix(qkv, heads, out_dtype):
    """qkv (P*4, 3H) = [q | k | v] -> (P*4, H)."""
    _rowmajor(qkv, "qkv")
    h = qkv.shape[1] // 3
    n_pos = qkv.shape[0] // 4
    out = torch.empty(n_pos * 4, h, dtype=out_dtype, device=qkv.device)
    es = qkv.element_size()
    call("mb_latent_mix", ptr(qkv), qkv.data_ptr() + h * es, qkv.data_ptr() + 2 * h * es, qkv.stride(0),
         dtype_code(qkv.dtype), n_pos, heads, h // heads, ptr(out), dtype_code(out_dtype), stream_of(qkv.device))
    return out


def layer_norm(x, gamma, beta, out_dtype=None, out=None, rows=None, eps=1e-5):
    _rowmajor(x, "x")
    n = rows.shape[0] if rows is not None else x.shape[0]
    h = x.shape[1]
    if out is None:
        out = torch.empty(n, h, dtype=out_dtype or x.dtype, device=x.device)
    call("mb_layer_norm", ptr(x), dtype_code(x.dtype), x.stride(0), ptr(rows), n, h, ptr(gamma), ptr(beta),
         float(eps), ptr(out), dtype_code(out.dtype), out.stride(0), stream_of(x.device))
    return out


def add_ln(x, y=None, y_bias=None, outs=(), eps=1e-5):
    """x += y (+ y_bias) in place, then LN_j(x) into each of ``outs``: a list of
    (gamma, beta, out tensor) with up to three entries (out views allowed)."""
    _rowmajor(x, "x")
    if len(outs) > 3:
        raise ValueError("add_ln takes at most three LayerNorm outputs")
    if y is not None:
        _rowmajor(y, "y")
    args = []
    for j in range(3):
        if j < len(outs):
            g, b, o = outs[j]
            _rowmajor(o, "out")
            args += [ptr(g), ptr(b), ptr(o), dtype_code(o.dtype), o.stride(0)]
        else:
            args += [None, None, None, 0, 0]
    call("mb_add_ln", ptr(x), x.stride(0), ptr(y), dtype_code(y.dtype) if y is not None else 0,
         y.stride(0) if y is not None else 0, ptr(y_bias), x.shape[0], x.shape[1], float(eps), *args,
         stream_of(x.device))
    return [o for _, _, o in outs]


def embed(ta, ia, tb=None, ib=None, n=None):
    n = n if n is not None else ia.shape[0]
    h = ta.shape[1]
    out = torch.empty(n, h, dtype=torch.float32, device=ta.device)
    call("mb_embed", ptr(ta), ta.shape[0], ptr(ia), ptr(tb), tb.shape[0] if tb is not None else 0, ptr(ib), n, h,
         ptr(out), stream_of(ta.device))
    return out


def cell_init(cov_ptr, cell_nearest, nearest_table, covered_row, covered_add=None):
    n, h = cell_nearest.shape[0], nearest_table.shape[1]
    out = torch.empty(n, h, dtype=torch.float32, device=nearest_table.device)
    call("mb_cell_init", ptr(cov_ptr), ptr(cell_nearest), ptr(nearest_table), nearest_table.shape[0],
         ptr(covered_row), ptr(covered_add), n, h, ptr(out), stream_of(out.device))
    return out


def residual_add(x, y, rows=None):
    """x[rows[i]] += y[i] (x f32 or bf16, in place)."""
    _rowmajor(x, "x"); _rowmajor(y, "y")
    n = y.shape[0]
    call("mb_residual_add", ptr(x), dtype_code(x.dtype), x.stride(0), ptr(rows), ptr(y), dtype_code(y.dtype),
         y.stride(0), n, y.shape[1], stream_of(x.device))
    return x


def add_gather(x, t, idx, relu=False):
    """x[i] = act(x[i] + t[idx[i]]) in place."""
    _rowmajor(x, "x"); _rowmajor(t, "t")
    call("mb_add_gather", ptr(x), dtype_code(x.dtype), x.stride(0), ptr(t), dtype_code(t.dtype), t.stride(0),
         t.shape[0], ptr(idx), x.shape[0], x.shape[1], int(relu), stream_of(x.device))
    return x


def tokens_gather(g, s, stone_off, tok_off, n_tok):
    h = g.shape[1]
    tok = torch.empty(n_tok, h, dtype=torch.float32, device=g.device)
    call("mb_tokens_gather", ptr(g), ptr(s), ptr(stone_off), ptr(tok_off), tok_off.shape[0] - 1, h, ptr(tok),
         stream_of(g.device))
    return tok


def tokens_scatter_add(g, s, stone_off, tok_off, tok_out, update_stones=True):
    call("mb_tokens_scatter_add", ptr(g), ptr(s), ptr(stone_off), ptr(tok_off), tok_off.shape[0] - 1, g.shape[1],
         ptr(tok_out), dtype_code(tok_out.dtype), int(update_stones), stream_of(g.device))


def latent_mean(g_ln, n_pos):
    h = g_ln.shape[1]
    out = torch.empty(n_pos, h, dtype=torch.float32, device=g_ln.device)
    call("mb_latent_mean", ptr(g_ln), n_pos, h, ptr(out), stream_of(g_ln.device))
    return out


def value_head(g, w, win_off, win_order, window_slot, value_valid, ln_g, ln_b, queries, w1, b1, w2, b2, centers,
               eps=1e-5):
    """(value (P,), value_dist (P, bins), value_logits (P, bins)) of the
    full forward's value readout (reference model.py:1160-1183) in one
    kernel: g (P, h) fp32 token rows, w (N_w, h) window rows (fp32 or bf16),
    the windows of position p at win_order[win_off[p]:win_off[p+1]]."""
    _cuda(g, w, win_off, window_slot, value_valid, queries, w1, w2)
    _rowmajor(g, "g")
    _rowmajor(w, "w")
    for t, n in ((win_off, "win_off"), (window_slot, "window_slot")):
        _i64(t, n)
    if win_order is not None:
        _i64(win_order, "win_order")
    p, h = g.shape
    nq = queries.shape[0]
    vh, bins = w1.shape[0], w2.shape[0]
    if w1.shape[1] != nq * h or w2.shape[1] != vh:
        raise ValueError("value head weights do not match the queries and width")
    f = lambda t: t.float().contiguous()
    vv = value_valid.to(torch.bool).contiguous()
    value = torch.empty(p, dtype=torch.float32, device=g.device)
    dist = torch.empty(p, bins, dtype=torch.float32, device=g.device)
    logits = torch.empty(p, bins, dtype=torch.float32, device=g.device)
    call("mb_value_head", ptr(g), ptr(w), dtype_code(w.dtype), w.stride(0), w.shape[0], ptr(win_off), ptr(win_order),
         ptr(window_slot), ptr(vv), p, vv.shape[1], h, ptr(f(ln_g)), ptr(f(ln_b)), float(eps), ptr(f(queries)), nq,
         ptr(f(w1)), ptr(f(b1)), vh, ptr(f(w2)), ptr(f(b2)), bins, ptr(f(centers)), ptr(value), ptr(dist),
         ptr(logits), stream_of(g.device))
    return value, dist, logits


def compose(critic, offsets, mass_floor):
    """(q_score, q_values) from (N, 3) fp32 logits (model.py:177-220)."""
    critic = critic.float()
    _rowmajor(critic, "critic")
    n = critic.shape[0]
    q_score = torch.empty(n, dtype=torch.float32, device=critic.device)
    q_values = torch.empty_like(q_score)
    call("mb_compose_q", ptr(critic), critic.stride(0), ptr(offsets), offsets.shape[0] - 1, float(mass_floor),
         ptr(q_score), ptr(q_values), stream_of(critic.device))
    return q_score, q_values


def linear_native(a, w, bias=None, relu=False, out_dtype=None, out=None):
    """CUDA-core GEMM with fp32 accumulation: act(a @ w^T + bias)."""
    _rowmajor(a, "a")
    w = w.contiguous()
    m, k = a.shape
    n = w.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=out_dtype or a.dtype, device=a.device)
    b = bias.float().contiguous() if bias is not None else None
    call("mb_linear", ptr(a), dtype_code(a.dtype), a.stride(0), m, k, ptr(w), dtype_code(w.dtype), ptr(b), n,
         int(relu), ptr(out), dtype_code(out.dtype), out.stride(0), stream_of(a.device))
    return out


# ================================================= reference op surface

class CellTables(NamedTuple):
    """cell_latents.py:78-93 (same field order and meaning)."""

    covered: torch.Tensor
    cell_ptr: torch.Tensor
    edge_window: torch.Tensor
    edge_class: torch.Tensor
    edge_cell: torch.Tensor
    win_ptr: torch.Tensor
    edge_wcell: torch.Tensor
    edge_wclass: torch.Tensor
    edge_wwin: torch.Tensor
    cls_ptr: torch.Tensor
    cedge_cell: torch.Tensor
    cedge_win: torch.Tensor


class IncidencePlan(NamedTuple):
    run_stone: torch.Tensor
    run_window: torch.Tensor
    run_class: torch.Tensor


def incidence_plan(inc_stone, inc_window, inc_class) -> IncidencePlan:
    """message_passing.py:495-517: the stone-major stable view."""
    if inc_class.shape != inc_stone.shape or inc_class.dtype != _I64:
        raise ValueError("inc_class must be int64 and one length with inc_stone")
    _cuda(inc_stone, inc_window, inc_class)
    bound = int(inc_stone.max().item()) + 1 if inc_stone.numel() else 1
    sk, order = argsort(inc_stone, bound)
    return IncidencePlan(sk, gather_i64(inc_window, order), gather_i64(inc_class, order))


def _covered_from_ptr(p: torch.Tensor) -> torch.Tensor:
    return torch.nonzero(p[1:] > p[:-1]).reshape(-1)


def cell_tables(dec_cell, dec_window, dec_class, n_windows, n_classes, n_cells=-1) -> CellTables:
    """cell_latents.py:96-165 on the device; bit-exact with the reference."""
    if not (dec_cell.shape == dec_window.shape == dec_class.shape):
        raise ValueError("dec_cell, dec_window, and dec_class must be one length")
    if dec_cell.ndim != 1:
        raise ValueError("decoder incidence arrays must be one-dimensional")
    _cuda(dec_cell, dec_window, dec_class)
    if dec_window.numel():
        if int(dec_window.min()) < 0 or int(dec_window.max()) >= n_windows:
            raise ValueError(f"dec_window entries must lie in [0, {n_windows})")
        if int(dec_class.min()) < 0 or int(dec_class.max()) >= n_classes:
            raise ValueError(f"dec_class entries must lie in [0, {n_classes})")
    bound = n_cells if n_cells >= 0 else (int(dec_cell.max()) + 1 if dec_cell.numel() else 1)
    if n_cells >= 0 and dec_cell.numel() and (int(dec_cell.min()) < 0 or int(dec_cell.max()) >= n_cells):
        raise ValueError(f"dec_cell entries must lie in [0, {n_cells})")
    sorted_cell, order = argsort(dec_cell, max(bound, 1))
    edge_window = gather_i64(dec_window, order)
    edge_class = gather_i64(dec_class, order)
    full_ptr = csr(sorted_cell, max(bound, 0))
    covered = _covered_from_ptr(full_ptr)
    if n_cells < 0:
        cell_ptr = torch.cat([full_ptr[covered], full_ptr[-1:]])
        compact = torch.cumsum((full_ptr[1:] > full_ptr[:-1]).to(_I64), 0) - 1
        edge_cell = gather_i64(compact, sorted_cell)
    else:
        cell_ptr = full_ptr
        edge_cell = sorted_cell
    win_sorted, worder = argsort(edge_window, max(n_windows, 1))
    win_ptr = csr(win_sorted, n_windows)
    cls_sorted, cedge_cell = argsort(edge_class, max(n_classes, 1))
    _, cedge_win = argsort(gather_i64(edge_class, worder), max(n_classes, 1))
    cls_ptr = csr(cls_sorted, n_classes)
    return CellTables(covered, cell_ptr, edge_window, edge_class, edge_cell, win_ptr, gather_i64(edge_cell, worder),
                      gather_i64(edge_class, worder), win_sorted, cls_ptr, cedge_cell, cedge_win)


def edge_tables(src, dst, cls, covered_destinations, n_sources, n_destinations, n_classes,
                uncovered_only) -> CellTables:
    """cell_nodes.py:23-94 on the device; bit-exact with the reference."""
    if not (src.shape == dst.shape == cls.shape) or src.ndim != 1:
        raise ValueError("src, dst, and cls must be one-dimensional and one length")
    _cuda(src, dst, cls, covered_destinations)
    if src.numel():
        if int(src.min()) < 0 or int(src.max()) >= n_sources:
            raise ValueError(f"src entries must lie in [0, {n_sources})")
        if int(dst.min()) < 0 or int(dst.max()) >= n_destinations:
            raise ValueError(f"dst entries must lie in [0, {n_destinations})")
        if int(cls.min()) < 0 or int(cls.max()) >= n_classes:
            raise ValueError(f"cls entries must lie in [0, {n_classes})")
    if uncovered_only:
        keep = ~torch.isin(dst, covered_destinations)
        src, dst, cls = src[keep], dst[keep], cls[keep]
    dst_sorted, order = argsort(dst, max(n_destinations, 1))
    edge_src = gather_i64(src, order)
    edge_class = gather_i64(cls, order)
    covered = torch.unique_consecutive(dst_sorted)
    dst_ptr = csr(dst_sorted, n_destinations)
    src_sorted, sorder = argsort(edge_src, max(n_sources, 1))
    src_ptr = csr(src_sorted, n_sources)
    edge_sclass = gather_i64(edge_class, sorder)
    cls_sorted, cedge_dst = argsort(edge_class, max(n_classes, 1))
    _, cedge_src = argsort(edge_sclass, max(n_classes, 1))
    cls_ptr = csr(cls_sorted, n_classes)
    return CellTables(covered, dst_ptr, edge_src, edge_class, dst_sorted, src_ptr, gather_i64(dst_sorted, sorder),
                      edge_sclass, src_sorted, cls_ptr, cedge_dst, cedge_src)


def window_latent_layout(window_pos, positions):
    """window_latents.py:38-56: position CSR offsets and stable order."""
    if window_pos.ndim != 1:
        raise ValueError("window_pos must have shape (N_w,)")
    if positions < 0:
        raise ValueError("positions must be nonnegative")
    _cuda(window_pos)
    if window_pos.numel():
        lo, hi = int(window_pos.min()), int(window_pos.max())
        if lo < 0 or hi >= positions:
            raise ValueError("window_pos entries must be in [0, positions)")
    sk, order = argsort(window_pos, max(positions, 1))
    return csr(sk, positions), order


def _validate_agg(values, inc_stone, inc_window, run_stone, run_window, n_dest):
    if values.ndim != 2:
        raise ValueError("values must have shape (N, H)")
    idx = (inc_stone, inc_window, run_stone, run_window)
    if inc_stone.ndim != 1 or any(i.shape != inc_stone.shape for i in idx):
        raise ValueError("the incidence views must be one length")
    if any(i.dtype != _I64 for i in idx):
        raise ValueError("incidence tensors must have dtype int64")
    if not values.is_floating_point():
        raise ValueError("values must have floating-point dtype")
    if n_dest < 0:
        raise ValueError(f"destination count must be nonnegative, got {n_dest}")
    _cuda(values, *idx)


def aggregate_to_windows(values, inc_stone, inc_window, run_stone, run_window, n_windows):
    """message_passing.py:283-297: sum stone rows into windows, output in values.dtype."""
    _validate_agg(values, inc_stone, inc_window, run_stone, run_window, n_windows)
    return run_reduce(values.contiguous(), inc_stone, csr(inc_window, n_windows), n_windows, out_dtype=values.dtype)


def aggregate_to_stones(values, inc_stone, inc_window, run_stone, run_window, n_stones):
    """message_passing.py:300-320: sum window rows into stones, fp32."""
    _validate_agg(values, inc_stone, inc_window, run_stone, run_window, n_stones)
    return run_reduce(values.contiguous(), run_window, csr(run_stone, n_stones), n_stones, out_dtype=torch.float32)


def class_row_sum(weight, gather, runs, n_dest, run_len=18):
    """message_passing.py:444-458: fp32 class-row sums per destination run."""
    if gather.ndim != 1 or gather.shape != runs.shape:
        raise ValueError("the incidence views must be one-dimensional and one length")
    if gather.dtype != _I64 or runs.dtype != _I64:
        raise ValueError("incidence tensors must have dtype int64")
    if n_dest < 0:
        raise ValueError(f"destination count must be nonnegative, got {n_dest}")
    _cuda(weight, gather, runs)
    w = weight.float().contiguous()
    return run_reduce(w, gather, csr(runs, n_dest), n_dest, out_dtype=torch.float32)


def incidence_row_sum(values, gather, runs, rev_gather, rev_runs, n_dest, run_len=18, rev_run_len=6):
    """message_passing.py:461-484 (forward): fp32 row sums per destination."""
    views = (gather, runs, rev_gather, rev_runs)
    if gather.ndim != 1 or any(v.shape != gather.shape for v in views):
        raise ValueError("the incidence views must be one-dimensional and one length")
    if any(v.dtype != _I64 for v in views):
        raise ValueError("incidence tensors must have dtype int64")
    _cuda(values, *views)
    return run_reduce(values.contiguous(), gather, csr(runs, n_dest), n_dest, out_dtype=torch.float32)


def _validate_cell_attention(q, k, v, bias, seg_ptr, src, cls, qid, sseg_ptr, sqid, scls):
    if q.ndim != 3 or k.shape != v.shape or q.shape[1:] != k.shape[1:]:
        raise ValueError("q and k/v must share (heads, head_dim)")
    if bias.ndim != 2 or bias.shape[0] != q.shape[1]:
        raise ValueError("bias must have shape (heads, classes)")
    if seg_ptr.numel() != q.shape[0] + 1:
        raise ValueError("seg_ptr must have one entry per query row plus one")
    if sseg_ptr.numel() != k.shape[0] + 1:
        raise ValueError("sseg_ptr must have one entry per source row plus one")
    if any(t.shape != src.shape for t in (cls, qid, sqid, scls)) or src.ndim != 1:
        raise ValueError("the edge views must have one length")
    _cuda(q, k, v, bias, seg_ptr, src, cls)


def cell_attention(q, k, v, bias, vcls, seg_ptr, src, cls, qid, sseg_ptr, sqid, scls, cptr, cedge_q):
    """cell_latents.py:834-856: (out fp32 (n_q, A, d), m, l)."""
    _validate_cell_attention(q, k, v, bias, seg_ptr, src, cls, qid, sseg_ptr, sqid, scls)
    if vcls.shape != (bias.shape[1], q.shape[1] * q.shape[2]):
        raise ValueError("vcls must have shape (classes, heads * head_dim)")
    out, m, l = segment_attention(q.contiguous(), k.contiguous(), v.contiguous(), bias, vcls, seg_ptr, src, cls,
                                  stats=True)
    return out.view(q.shape), m, l


def cell_attention_plain(q, k, v, bias, seg_ptr, src, cls, qid, sseg_ptr, sqid, scls, cptr, cedge_q):
    """cell_latents.py:922-940: score bias only."""
    _validate_cell_attention(q, k, v, bias, seg_ptr, src, cls, qid, sseg_ptr, sqid, scls)
    out, m, l = segment_attention(q.contiguous(), k.contiguous(), v.contiguous(), bias, None, seg_ptr, src, cls,
                                  stats=True)
    return out.view(q.shape), m, l


def read_attention(q, k, v, window_pos, offsets, order):
    """window_latents.py:717-720: (P, 4, A, d) latent queries over windows, fp32."""
    if q.ndim != 4 or q.shape[1] != 4:
        raise ValueError("read q must have shape (P, 4, heads, head_dim)")
    if k.ndim != 3 or k.shape != v.shape or q.shape[2:] != k.shape[1:]:
        raise ValueError("read q, k, and v must share heads and head_dim")
    _cuda(q, k, v, offsets, order)
    p, _, heads, hd = q.shape
    out = latent_read(q.reshape(p * 4, -1).contiguous(), k.reshape(k.shape[0], -1).contiguous(),
                      v.reshape(v.shape[0], -1).contiguous(), heads, offsets, order)
    return out.view(q.shape)


def broadcast_attention(q, k, v, window_pos, offsets, order):
    """window_latents.py:723-726: windows over their position's 4 latents, fp32."""
    if q.ndim != 3 or k.ndim != 4 or k.shape != v.shape or k.shape[1] != 4 or q.shape[1:] != k.shape[2:]:
        raise ValueError("broadcast q (N_w, A, d) and k/v (P, 4, A, d) shapes disagree")
    _cuda(q, k, v, window_pos)
    n_w, heads, hd = q.shape
    out = latent_broadcast(q.reshape(n_w, -1).contiguous(), k.reshape(-1, heads * hd).contiguous(),
                           v.reshape(-1, heads * hd).contiguous(), heads, window_pos, k.shape[0])
    return out.view(q.shape)


def encode_rows(pre_w, table, edge_window, edge_class, edge_cell, edge_rev, n_cells):
    """row_encoder.py:416-447: fp32 sum of relu(pre_w[window] + table[class]) per cell."""
    views = (edge_window, edge_class, edge_cell, edge_rev)
    if any(v.shape != edge_window.shape for v in views) or edge_window.ndim != 1:
        raise ValueError("edge views must be one-dimensional and one length")
    _cuda(pre_w, table, *views)
    return row_encode(pre_w.contiguous(), table.float().contiguous(), edge_window, edge_class,
                      csr(edge_cell, n_cells), n_cells)


def cell_pass(x, emb, cell_ptr, edge_window, edge_class, win_ptr, edge_wcell, cls_ptr, edge_ccell):
    """relay.py:577-591: the (N_w, H) window aggregate, in x's dtype."""
    _cuda(x, emb, cell_ptr, edge_window, edge_class, win_ptr, edge_wcell)
    n_cov = cell_ptr.numel() - 1
    h = x.shape[1]
    x = x.contiguous()
    out = torch.empty_like(x)
    scratch = torch.empty(max(n_cov, 1), h, dtype=torch.float32, device=x.device)
    e = emb.float().contiguous()
    call("mb_cell_pass", ptr(x), dtype_code(x.dtype), x.shape[0], ptr(e), e.shape[0], ptr(cell_ptr), n_cov,
         ptr(edge_window), ptr(edge_class), ptr(win_ptr), ptr(edge_wcell), h, ptr(scratch), ptr(out),
         dtype_code(out.dtype), stream_of(x.device))
    return out


def fused_attention(q, k, v, seq_lens, with_lse: bool = False):
    """attention.py:892-904: block-diagonal attention over (P, A, T, D)
    (strided views allowed, inner stride 1); keys >= seq_lens[p] masked, pad
    query rows zero. Output preserves q's strides like ``empty_like``. With
    ``with_lse`` also the per-row log-sum-exp of the scaled scores (P, A, T)
    fp32, 0 on pad rows (the op's auxiliary output, attention.py:155-162)."""
    if q.ndim != 4 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k, and v must have the same (P, A, T, D) shape")
    p, heads, t, d = q.shape
    if seq_lens.shape != (p,) or seq_lens.dtype != torch.int32:
        raise ValueError("seq_lens must be int32 with shape (P,)")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k, and v must have one dtype")
    _cuda(q, k, v, seq_lens)
    if not (q.stride() == k.stride() == v.stride()) or q.stride(3) != 1:
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    out = torch.empty_like(q)
    lse = torch.empty(p, heads, t, dtype=torch.float32, device=q.device) if with_lse else None
    sp, sa, st, _ = q.stride()
    op, oa, ot, _ = out.stride()
    call("mb_stone_attention", ptr(q), ptr(k), ptr(v), dtype_code(q.dtype), p, heads, d, sp, sa, st,
         ptr(seq_lens.contiguous()), t, None, 0, -1, ptr(out), dtype_code(out.dtype), op, oa, ot, ptr(lse),
         stream_of(q.device))
    return (out, lse) if with_lse else out


# ============================================ tcgen05 fused row GEMM (sm_100a)

GEMM_K = GEMM_N = 256
GEMM_KS = (256, 512)  # the K widths the tensor-core row GEMM holds whole in shared memory


def weight_image(w: torch.Tensor) -> torch.Tensor:
    """The pre-swizzled bf16 image of an (N, K) weight for ``gemm_rows``:
    N a multiple of 128, K 256 or 512."""
    _cuda(w)
    w = w.detach().to(torch.bfloat16).contiguous()
    n, k = w.shape
    if n % 128 or n == 0 or k not in GEMM_KS:
        raise ValueError(f"gemm weight must be (N, K) with N a multiple of 128 and K in {GEMM_KS}, got {(n, k)}")
    img = torch.empty_like(w)
    call("mb_gemm_weight_image", ptr(w), n, k, ptr(img), stream_of(w.device))
    return img


def gemm_rows(x, w_img, bias=None, gamma=None, beta=None, relu=False, out=None, residual=None, eps=1e-5, add=None):
    """act(prologue(x) @ W^T + bias (+ add)) on tcgen05: LayerNorm prologue
    when ``gamma`` is given (x fp32, width 256), else x bf16 (width 256 or
    512). ``w_img`` is ``weight_image(W)`` of W (N, K); N is read from it.
    Writes ``out`` (bf16, allocated when neither out nor residual is given),
    optionally plus fp32 addend rows ``add``, or adds into ``residual``
    (fp32, N = 256)."""
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be 2-D with unit column stride")
    m, k = x.shape
    n = w_img.shape[0]
    if w_img.shape[1] != k:
        raise ValueError(f"x width {k} does not match the weight's K {w_img.shape[1]}")
    if out is None and residual is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    if out is not None and (out.dtype != torch.bfloat16 or out.shape != (m, n) or out.stride(1) != 1):
        raise ValueError("out must be (m, N) bf16 with unit column stride")
    if add is not None and (add.dtype != torch.float32 or add.shape != (m, n) or add.stride(1) != 1):
        raise ValueError("add must be (m, N) fp32 with unit column stride")
    b = bias.float().contiguous() if bias is not None else None
    call("mb_gemm_rows_ex", ptr(x), dtype_code(x.dtype), x.stride(0), m, k, ptr(gamma), ptr(beta), float(eps),
         ptr(w_img), n, ptr(b), int(relu), ptr(add), add.stride(0) if add is not None else 0, ptr(out),
         out.stride(0) if out is not None else 0, ptr(residual), residual.stride(0) if residual is not None else 0,
         stream_of(x.device))
    return out if out is not None else residual


def gemm_head(x, w_img, bias, tok, tok_idx, w_out, b_out, out=None):
    """A decoder head's hidden and output layers in one tensor-core launch
    (reference _PairMlp over a per-cell row and its position's row,
    model.py:246-260, 1031-1139):
        out[r] = relu(x[r] @ W^T + bias + tok[tok_idx[r]]) @ w_out^T + b_out
    x (m, 256) bf16; W (N, 256) with N 128 or 256; tok (P, N) bf16 rows (the
    position half lin_b(g), already projected); w_out (n_out, N) fp32 with
    n_out <= 4; out (m, n_out) fp32."""
    _rowmajor(x, "x")
    _rowmajor(tok, "tok")
    n = w_img.shape[0]
    n_out = w_out.shape[0]
    if x.dtype != torch.bfloat16 or tok.dtype != torch.bfloat16 or tok.shape[1] != n:
        raise ValueError("gemm_head takes bf16 x and bf16 tok rows of the hidden width")
    if out is None:
        out = torch.empty(x.shape[0], n_out, dtype=torch.float32, device=x.device)
    _i64(tok_idx, "tok_idx")
    if tok_idx.shape != (x.shape[0],):
        raise ValueError("tok_idx must hold one position per row")
    wo = w_out if (w_out.dtype == torch.float32 and w_out.is_contiguous()) else w_out.float().contiguous()
    bo = b_out if (b_out.dtype == torch.float32 and b_out.is_contiguous()) else b_out.float().contiguous()
    if out.dtype != torch.float32 or out.shape != (x.shape[0], n_out) or out.stride(1) != 1:
        raise ValueError("out must be (m, n_out) fp32 rows")
    call("mb_gemm_rows_head", ptr(x), x.stride(0), x.shape[0], ptr(w_img), n, ptr(bias), ptr(tok), tok.stride(0),
         tok.shape[0], ptr(tok_idx), ptr(wo), ptr(bo), n_out, ptr(out), out.stride(0), stream_of(x.device))
    return out


def gemm_rows_ln(a, w_img, bias, residual, outs, eps=1e-5):
    """residual += a @ W^T + bias (fp32 rows, in place), then one LayerNorm of
    each updated row per ``outs`` entry ``(gamma, beta, out)`` (out bf16, unit
    column stride, up to three), in one tcgen05 launch."""
    _rowmajor(a, "a")
    if a.dtype != torch.bfloat16 or a.shape[1] != GEMM_K:
        raise ValueError(f"gemm_rows_ln takes bf16 rows of width {GEMM_K}")
    if residual.dtype != torch.float32 or residual.shape != (a.shape[0], GEMM_N) or residual.stride(1) != 1:
        raise ValueError("residual must be (m, 256) fp32 rows")
    if len(outs) > 3:
        raise ValueError("at most three LayerNorm outputs")
    args = []
    for g, b, o in outs:
        if o.shape != residual.shape or o.stride(1) != 1 or o.dtype != torch.bfloat16:
            raise ValueError("LayerNorm outputs must be bf16 and match the residual's shape with unit column stride")
        args += [ptr(g), ptr(b), ptr(o), dtype_code(o.dtype), o.stride(0)]
    args += [None, None, None, 0, 0] * (3 - len(outs))
    bb = bias.float().contiguous() if bias is not None else None
    call("mb_gemm_rows_ln", ptr(a), a.stride(0), a.shape[0], ptr(w_img), ptr(bb), ptr(residual), residual.stride(0),
         float(eps), *args, stream_of(a.device))
    return [o for _, _, o in outs]


# ------------------------------------------------- isolated-op workloads
def hex_message_pass(x, nbr, w_img, bias=None, out=None):
    """out = x + W mean(x[present neighbours]) + bias, fused on the tensor
    cores. x (n, 256) bf16 rows; nbr (n, 6) int32 (-1 absent); w_img from
    ``weight_image(W)``; bias fp32 (256,) or None."""
    _cuda(x, nbr, w_img)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != GEMM_K or x.stride(1) != 1:
        raise ValueError("hex_message_pass takes (n, 256) bf16 rows")
    if nbr.dtype != torch.int32 or tuple(nbr.shape) != (x.shape[0], 6) or not nbr.is_contiguous():
        raise ValueError("nbr must be a contiguous (n, 6) int32 table")
    if bias is not None and (bias.dtype != torch.float32 or bias.numel() != GEMM_N or not bias.is_contiguous()):
        raise ValueError("bias must be a contiguous fp32 (256,) vector")
    if out is None:
        out = torch.empty(x.shape[0], GEMM_N, dtype=torch.bfloat16, device=x.device)
    call("mb_hex_message_pass", ptr(x), x.stride(0), x.shape[0], ptr(nbr), ptr(w_img), ptr(bias), ptr(out),
         out.stride(0), stream_of(x.device))
    return out


def axial_attention(q, k, v, coords, valid, bias, out=None):
    """Cell-token attention with the (dq, dr) relative-offset bias. q/k/v
    (P, H, L, 32) bf16 (any strides with unit last stride, 16-byte aligned
    rows); coords (P, L, 2) int32; valid (P,) int32; bias (33, 33, H) fp32.
    Returns (P, H, L, 32) bf16 with rows past valid[p] zero."""
    _cuda(q, k, v, coords, valid, bias)
    if not (q.shape == k.shape == v.shape) or q.dim() != 4 or q.dtype != torch.bfloat16:
        raise ValueError("q, k and v must be (P, H, L, d) bf16 of one shape")
    if not (q.stride() == k.stride() == v.stride()) or q.stride(3) != 1:
        raise ValueError("q, k and v must share strides with a unit last stride")
    p, h, length, d = q.shape
    if coords.dtype != torch.int32 or tuple(coords.shape) != (p, length, 2) or not coords.is_contiguous():
        raise ValueError("coords must be a contiguous (P, L, 2) int32 tensor")
    if valid.dtype != torch.int32 or tuple(valid.shape) != (p,):
        raise ValueError("valid must be a (P,) int32 tensor")
    if bias.dtype != torch.float32 or tuple(bias.shape) != (33, 33, h) or not bias.is_contiguous():
        raise ValueError("bias must be a contiguous (33, 33, H) fp32 table")
    if out is None:
        out = torch.empty(p, h, length, d, dtype=torch.bfloat16, device=q.device)
    call("mb_axial_attention", ptr(q), ptr(k), ptr(v), p, h, d, length, q.stride(0), q.stride(1), q.stride(2),
         ptr(coords), ptr(valid), ptr(bias), ptr(out), out.stride(0), out.stride(1), out.stride(2),
         stream_of(q.device))
    return out


# ----------------------------------------------------- KLENT improvement
class ImprovedPolicy(NamedTuple):
    """pi' and its per-position diagnostics, flat over the legal cells
    (reference klent/improve.py:18-24)."""
    probs: torch.Tensor
    v_hat: torch.Tensor
    kl: torch.Tensor
    norm_entropy: torch.Tensor


class Draw(NamedTuple):
    """The self-play move draw (reference klent/selfplay.py:180-190)."""
    stored: torch.Tensor     # (N,) float32 pi' renormalised in float64
    ranks: torch.Tensor      # (P,) int64 chosen legal-cell rank
    pi_top1: torch.Tensor    # (P,) float64
    pi_chosen: torch.Tensor  # (P,) float64


def improved_policy(policy_logits, q_score, q_value, offsets, tau, lam, uniforms=None):
    """klent/improve.py:27-69 on the device (float32 inputs; sums in float64).
    With ``uniforms`` (one float64 in [0, 1) per position) also the move draw:
    returns (ImprovedPolicy, Draw), else the ImprovedPolicy."""
    if tau < 0 or lam < 0 or tau + lam <= 0:
        raise ValueError(f"need tau, lam >= 0 with tau + lam > 0, got ({tau}, {lam})")
    if q_score.shape != q_value.shape:
        raise ValueError("q_score and q_value must have the same shape, got "
                         f"{tuple(q_score.shape)} and {tuple(q_value.shape)}")
    _cuda(policy_logits, q_score, q_value, offsets)
    if policy_logits.shape != q_score.shape or policy_logits.dim() != 1:
        raise ValueError("policy_logits, q_score and q_value must be one-dimensional and one length")
    if offsets.dtype != _I64 or offsets.dim() != 1 or offsets.shape[0] < 1:
        raise ValueError("offsets must be a (P + 1,) int64 tensor")
    x, sc, q = (t.float().contiguous() for t in (policy_logits, q_score, q_value))
    off = offsets.contiguous()
    n, p = x.shape[0], off.shape[0] - 1
    dev = x.device
    probs = torch.empty(n, dtype=torch.float32, device=dev)
    v_hat, kl, ne = (torch.empty(p, dtype=torch.float32, device=dev) for _ in range(3))
    draw = None
    if uniforms is not None:
        u = uniforms.to(device=dev, dtype=torch.float64).contiguous()
        if u.shape != (p,):
            raise ValueError(f"uniforms must hold one draw per position ({p})")
        draw = Draw(torch.empty(n, dtype=torch.float32, device=dev), torch.empty(p, dtype=torch.int64, device=dev),
                    torch.empty(p, dtype=torch.float64, device=dev), torch.empty(p, dtype=torch.float64, device=dev))
    call("mb_klent_improve", ptr(x), ptr(sc), ptr(q), ptr(off), p, n, float(tau), float(lam), ptr(probs), ptr(v_hat),
         ptr(kl), ptr(ne), ptr(u) if draw else None, ptr(draw.stored) if draw else None,
         ptr(draw.ranks) if draw else None, ptr(draw.pi_top1) if draw else None,
         ptr(draw.pi_chosen) if draw else None, stream_of(dev))
    imp = ImprovedPolicy(probs, v_hat, kl, ne)
    return (imp, draw) if draw is not None else imp


def segment_argmax(x, offsets):
    """Per segment of ``x`` (cut by ``offsets``), the rank of its largest
    value, the first on ties (-1 for an empty segment): (P,) int64."""
    _cuda(x, offsets)
    _i64(offsets, "offsets")
    xf = x.float().contiguous()
    p = offsets.shape[0] - 1
    ranks = torch.empty(p, dtype=torch.int64, device=x.device)
    call("mb_segment_argmax", ptr(xf), ptr(offsets), p, xf.shape[0], ptr(ranks), stream_of(x.device))
    return ranks


# ============================================================ backward
# Deterministic gradients of the data-dependent ops (no atomics): the edge
# permutations by source / class / window come from the stable device sort.
def _perm_csr(keys, bound):
    """(stable order of ``keys``, CSR of the sorted keys over [0, bound))."""
    sk, order = argsort(keys, max(int(bound), 1))
    return order, csr(sk, bound)


def segment_attention_backward(q, k, v, bias, vcls, seg_ptr, src, cls, m, l, grad_out, qid=None):
    """Gradients of ``segment_attention`` (typed segment attention; the
    reference's cell_attention_backward, cell_latents.py:869-990): q (n_q, H)
    or (n_q, A, d) rows, k / v likewise, m / l (n_q, A) from the forward,
    grad_out like the output. Returns (dq, dk, dv, dbias, dvcls or None) in
    the dtypes of q, k, v, bias, vcls."""
    _cuda(q, k, v, bias, seg_ptr, src, cls, m, l, grad_out)
    heads = bias.shape[0]
    n_q, n_src = q.shape[0], k.shape[0]
    H = q[0].numel() if n_q else k[0].numel()
    hd = H // heads
    n_cls = bias.shape[1]
    qc, kc, vc = (t.reshape(t.shape[0], H).contiguous() for t in (q, k, v))
    if not (qc.dtype == kc.dtype == vc.dtype):
        raise ValueError("q, k and v must have one dtype")
    go = grad_out.reshape(n_q, H).float().contiguous()
    e = src.shape[0]
    if qid is None:
        qid = torch.repeat_interleave(torch.arange(n_q, device=q.device), seg_ptr[1:] - seg_ptr[:-1])
    src_perm, src_ptr = _perm_csr(src, n_src)
    cls_perm, cls_ptr = _perm_csr(cls, n_cls)
    ws_a = torch.empty(max(e, 1), heads, dtype=torch.float32, device=q.device)
    ws_d = torch.empty_like(ws_a)
    dq = torch.empty(n_q, H, dtype=torch.float32, device=q.device)
    dk = torch.empty(n_src, H, dtype=torch.float32, device=q.device)
    dv = torch.empty_like(dk)
    dbias = torch.empty(heads, n_cls, dtype=torch.float32, device=q.device)
    vcl = None if vcls is None else vcls.reshape(n_cls, H).contiguous()
    dvcls = None if vcls is None else torch.empty(n_cls, H, dtype=torch.float32, device=q.device)
    b32 = bias.float().contiguous()
    call("mb_segment_attention_backward", ptr(qc), ptr(kc), ptr(vc), dtype_code(qc.dtype), n_q, n_src, heads, hd,
         ptr(b32), n_cls, ptr(vcl), dtype_code(vcl.dtype) if vcl is not None else 0, ptr(seg_ptr), ptr(src),
         ptr(cls), ptr(qid.contiguous()), ptr(m.float().contiguous()), ptr(l.float().contiguous()), ptr(go), e,
         ptr(src_perm), ptr(src_ptr), ptr(cls_perm), ptr(cls_ptr), ptr(ws_a), ptr(ws_d), ptr(dq), ptr(dk), ptr(dv),
         ptr(dbias), ptr(dvcls), stream_of(q.device))
    out = (dq.view(q.shape).to(q.dtype), dk.view(k.shape).to(k.dtype), dv.view(v.shape).to(v.dtype),
           dbias.to(bias.dtype), None if vcls is None else dvcls.view(vcls.shape).to(vcls.dtype))
    return out


def stone_attention_backward(q, k, v, seq_lens, out, lse, grad_out):
    """Gradients of ``fused_attention`` (the reference's
    fused_attention_backward, attention.py:823-890) on the padded (P, A, T, D)
    layout with the forward's ``lse``: (dq, dk, dv) in q's dtype."""
    _cuda(q, k, v, seq_lens, out, lse, grad_out)
    p, heads, t, d = q.shape
    tens = [q, k, v, out, grad_out.to(q.dtype)]
    if not all(x.stride() == q.stride() for x in tens) or q.stride(3) != 1:
        tens = [x.contiguous() for x in tens]
    q_, k_, v_, o_, g_ = tens
    sp, sa, st, _ = q_.stride()
    dsum = torch.empty(p, heads, t, dtype=torch.float32, device=q.device)
    grads = [torch.empty(p, heads, t, d, dtype=torch.float32, device=q.device) for _ in range(3)]
    call("mb_stone_attention_backward", ptr(q_), ptr(k_), ptr(v_), ptr(o_), ptr(g_), dtype_code(q_.dtype), p, heads,
         d, sp, sa, st, ptr(seq_lens.contiguous()), t, ptr(lse.float().contiguous()), ptr(dsum), *map(ptr, grads),
         stream_of(q.device))
    return tuple(g.to(q.dtype) for g in grads)


def window_latent_read_backward(q, k, v, offsets, order, window_pos, out, m, l, grad_out):
    """Gradients of the window-latent read (reference
    window_latent_read_backward, window_latents.py:589-640): q (P, 4, A, d),
    k / v (N_w, A, d), out / m / l from the forward."""
    _cuda(q, k, v, offsets, window_pos, out, m, l, grad_out)
    p, _, heads, hd = q.shape
    n_w = k.shape[0]
    H = heads * hd
    qc, kc, vc = q.reshape(p * 4, H).contiguous(), k.reshape(n_w, H).contiguous(), v.reshape(n_w, H).contiguous()
    dq = torch.empty(p * 4, H, dtype=torch.float32, device=q.device)
    dk = torch.empty(n_w, H, dtype=torch.float32, device=q.device)
    dv = torch.empty_like(dk)
    call("mb_window_latent_read_backward", ptr(qc), ptr(kc), ptr(vc), dtype_code(qc.dtype),
         ptr(out.reshape(p * 4, H).float().contiguous()), ptr(m.float().contiguous()), ptr(l.float().contiguous()),
         ptr(grad_out.reshape(p * 4, H).float().contiguous()), ptr(window_pos.contiguous()), ptr(offsets),
         ptr(order), p, n_w, heads, hd, ptr(dq), ptr(dk), ptr(dv), stream_of(q.device))
    return dq.view(q.shape).to(q.dtype), dk.view(k.shape).to(k.dtype), dv.view(v.shape).to(v.dtype)


def window_latent_broadcast_backward(q, k, v, offsets, order, window_pos, m, l, grad_out):
    """Gradients of the window-latent broadcast (reference
    window_latent_broadcast_backward, window_latents.py:666-700): q (N_w, A,
    d), k / v (P, 4, A, d), m / l from the forward."""
    _cuda(q, k, v, offsets, window_pos, m, l, grad_out)
    n_w, heads, hd = q.shape
    p = k.shape[0]
    H = heads * hd
    qc, kc, vc = q.reshape(n_w, H).contiguous(), k.reshape(p * 4, H).contiguous(), v.reshape(p * 4, H).contiguous()
    ws = [torch.empty(max(n_w, 1), 4, heads, dtype=torch.float32, device=q.device) for _ in range(2)]
    dq = torch.empty(n_w, H, dtype=torch.float32, device=q.device)
    dk = torch.empty(p * 4, H, dtype=torch.float32, device=q.device)
    dv = torch.empty_like(dk)
    call("mb_window_latent_broadcast_backward", ptr(qc), ptr(kc), ptr(vc), dtype_code(qc.dtype),
         ptr(m.float().contiguous()), ptr(l.float().contiguous()), ptr(grad_out.reshape(n_w, H).float().contiguous()),
         ptr(window_pos.contiguous()), ptr(offsets), ptr(order), p, n_w, heads, hd, ptr(ws[0]), ptr(ws[1]), ptr(dq),
         ptr(dk), ptr(dv), stream_of(q.device))
    return dq.view(q.shape).to(q.dtype), dk.view(k.shape).to(k.dtype), dv.view(v.shape).to(v.dtype)


def encode_rows_backward(pre_w, table, edge_window, edge_class, edge_cell, grad_out):
    """Gradients of ``encode_rows`` (the action-row encoder,
    row_encoder.py:114-207): (grad_pre_w, grad_table) in their dtypes."""
    _cuda(pre_w, table, edge_window, edge_class, edge_cell, grad_out)
    n_pre, h = pre_w.shape
    n_table = table.shape[0]
    pc = pre_w.contiguous()
    t32 = table.float().contiguous()
    win_perm, win_ptr = _perm_csr(edge_window, n_pre)
    cls_perm, cls_ptr = _perm_csr(edge_class, n_table)
    gp = torch.empty(n_pre, h, dtype=torch.float32, device=pre_w.device)
    gt = torch.empty(n_table, h, dtype=torch.float32, device=pre_w.device)
    call("mb_row_encode_backward", ptr(pc), dtype_code(pc.dtype), n_pre, ptr(t32), n_table, ptr(edge_window),
         ptr(edge_class), ptr(edge_cell), edge_window.shape[0], ptr(grad_out.float().contiguous()),
         grad_out.shape[0], h, ptr(win_perm), ptr(win_ptr), ptr(cls_perm), ptr(cls_ptr), ptr(gp), ptr(gt),
         stream_of(pre_w.device))
    return gp.to(pre_w.dtype), gt.to(table.dtype)
