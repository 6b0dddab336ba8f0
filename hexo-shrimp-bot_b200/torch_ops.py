"""The operator-level plug-in: this library's kernels behind the reference's
``mantisnet::`` torch.library custom ops.

The reference registers each data-dependent forward of MantisNet as an
opaque custom op (e.g. python/mantisnet/mantisnet/attention.py:719-753,
cell_latents.py:834-860, window_latents.py:553-714, message_passing.py:191-365,
row_encoder.py:368-380, relay.py:452) with a ``register_fake`` so that
``torch.compile(dynamic=True, fullgraph=True)`` keeps it opaque. Two ways in:

- :func:`install_into_reference` registers a CUDA kernel of this library for
  every one of those ops that is already defined (the reference package
  imported), so the reference's own ``MantisNet`` runs its op calls on these
  kernels; the reference's fakes and CPU paths stay as they are.
- :func:`define` defines the same ops (names, argument lists, output
  contracts) in a namespace of their own (default ``mantis_b200``) with these
  kernels and fake implementations, for callers without the reference.

Backward: :func:`define` registers autograd for the attention ops and the
action-row encoder on this library's deterministic backward kernels, and
:func:`install_into_reference` also takes over the reference's backward ops
(``*_backward``, e.g. attention.py:823-890, cell_latents.py:869-990,
window_latents.py:589-700), so the reference's own autograd formulas call
these kernels. Every output follows the reference op's contract, auxiliary
statistics included (fused_attention's per-row log-sum-exp, the segment
attentions' running max and sum).
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import ops

# op name -> schema (the reference's argument names and types)
_SCHEMAS = {
    "fused_attention": "(Tensor q, Tensor k, Tensor v, Tensor seq_lens) -> (Tensor, Tensor)",
    "cell_attention": ("(Tensor q, Tensor k, Tensor v, Tensor bias, Tensor vcls, Tensor seg_ptr, Tensor src, "
                       "Tensor cls, Tensor qid, Tensor sseg_ptr, Tensor sqid, Tensor scls, Tensor cptr, "
                       "Tensor cedge_q) -> (Tensor, Tensor, Tensor)"),
    "cell_attention_plain": ("(Tensor q, Tensor k, Tensor v, Tensor bias, Tensor seg_ptr, Tensor src, Tensor cls, "
                             "Tensor qid, Tensor sseg_ptr, Tensor sqid, Tensor scls, Tensor cptr, Tensor cedge_q) "
                             "-> (Tensor, Tensor, Tensor)"),
    "window_latent_read": ("(Tensor q, Tensor k, Tensor v, Tensor window_pos, Tensor offsets, Tensor order) "
                           "-> (Tensor, Tensor, Tensor)"),
    "window_latent_broadcast": ("(Tensor q, Tensor k, Tensor v, Tensor window_pos, Tensor offsets, Tensor order) "
                                "-> (Tensor, Tensor, Tensor)"),
    "aggregate_to_windows": ("(Tensor values, Tensor inc_stone, Tensor inc_window, Tensor run_stone, "
                             "Tensor run_window, int n_windows) -> Tensor"),
    "aggregate_to_stones": ("(Tensor values, Tensor inc_stone, Tensor inc_window, Tensor run_stone, "
                            "Tensor run_window, int n_stones) -> Tensor"),
    "class_row_sum": "(Tensor weight, Tensor gather, Tensor runs, int n_dest, int run_len) -> Tensor",
    "incidence_row_sum": ("(Tensor values, Tensor gather, Tensor runs, Tensor rev_gather, Tensor rev_runs, "
                          "int n_dest, int run_len, int rev_run_len) -> Tensor"),
    "action_row_encode": ("(Tensor pre_w, Tensor table, Tensor edge_window, Tensor edge_class, Tensor edge_cell, "
                          "Tensor edge_rev, int n_cells) -> Tensor"),
    "cell_pass": ("(Tensor x, Tensor emb, Tensor cell_ptr, Tensor edge_window, Tensor edge_class, Tensor win_ptr, "
                  "Tensor edge_wcell, Tensor cls_ptr, Tensor edge_ccell) -> Tensor"),
    "window_latent_layout": "(Tensor window_pos, int positions) -> (Tensor, Tensor)",
}


def _lse_wanted(q: Tensor) -> bool:
    """The reference returns a (P, A, T) log-sum-exp when its CUDA kernel
    serves the shape (fp16 / bf16, head_dim 16, 32 or 64), else an empty one
    (attention.py:727-732, 756-772)."""
    return q.is_cuda and q.dtype in (torch.float16, torch.bfloat16) and q.shape[-1] in (16, 32, 64)


# ------------------------------------------------------------ CUDA kernels
def _fused_attention(q, k, v, seq_lens):
    if q.dtype == torch.float16:
        raise NotImplementedError("mantisnet::fused_attention on this library takes bf16 or fp32 tensors")
    if _lse_wanted(q):
        return ops.fused_attention(q, k, v, seq_lens, with_lse=True)
    return ops.fused_attention(q, k, v, seq_lens), torch.empty(0, dtype=torch.float32, device=q.device)


def _cell_attention(q, k, v, bias, vcls, seg_ptr, src, cls, qid, sseg_ptr, sqid, scls, cptr, cedge_q):
    return tuple(ops.cell_attention(q, k, v, bias, vcls, seg_ptr, src, cls, qid, sseg_ptr, sqid, scls, cptr, cedge_q))


def _cell_attention_plain(q, k, v, bias, seg_ptr, src, cls, qid, sseg_ptr, sqid, scls, cptr, cedge_q):
    return tuple(ops.cell_attention_plain(q, k, v, bias, seg_ptr, src, cls, qid, sseg_ptr, sqid, scls, cptr, cedge_q))


def _window_latent_read(q, k, v, window_pos, offsets, order):
    p, _, heads, hd = q.shape
    out, m, l = ops.latent_read(q.reshape(p * 4, -1).contiguous(), k.reshape(k.shape[0], -1).contiguous(),
                                v.reshape(v.shape[0], -1).contiguous(), heads, offsets, order, stats=True)
    return out.view(q.shape), m.view(q.shape[:-1]), l.view(q.shape[:-1])


def _window_latent_broadcast(q, k, v, window_pos, offsets, order):
    n_w, heads, hd = q.shape
    out, m, l = ops.latent_broadcast(q.reshape(n_w, -1).contiguous(), k.reshape(-1, heads * hd).contiguous(),
                                     v.reshape(-1, heads * hd).contiguous(), heads, window_pos, k.shape[0],
                                     stats=True)
    return out.view(q.shape), m.view(q.shape[:-1]), l.view(q.shape[:-1])


def _window_latent_layout(window_pos, positions):
    return tuple(ops.window_latent_layout(window_pos, positions))


_KERNELS = {
    "fused_attention": _fused_attention,
    "cell_attention": _cell_attention,
    "cell_attention_plain": _cell_attention_plain,
    "window_latent_read": _window_latent_read,
    "window_latent_broadcast": _window_latent_broadcast,
    "aggregate_to_windows": ops.aggregate_to_windows,
    "aggregate_to_stones": ops.aggregate_to_stones,
    "class_row_sum": ops.class_row_sum,
    "incidence_row_sum": ops.incidence_row_sum,
    "action_row_encode": ops.encode_rows,
    "cell_pass": ops.cell_pass,
    "window_latent_layout": _window_latent_layout,
}


# ------------------------------------------------------------- fakes
def _fake_fused_attention(q, k, v, seq_lens):
    lse = (q.new_empty(q.shape[:3], dtype=torch.float32) if _lse_wanted(q)
           else q.new_empty((0,), dtype=torch.float32))
    return torch.empty_like(q), lse


def _fake_segment(q, *rest):
    n_q, heads, hd = q.shape
    return (q.new_empty((n_q, heads, hd), dtype=torch.float32), q.new_empty((n_q, heads), dtype=torch.float32),
            q.new_empty((n_q, heads), dtype=torch.float32))


def _fake_latent(q, k, v, window_pos, offsets, order):
    return (q.new_empty(q.shape, dtype=torch.float32), q.new_empty(q.shape[:-1], dtype=torch.float32),
            q.new_empty(q.shape[:-1], dtype=torch.float32))


def _fake_aggregate_to_windows(values, inc_stone, inc_window, run_stone, run_window, n_windows):
    return values.new_empty((n_windows, values.shape[1]))


def _fake_aggregate_to_stones(values, inc_stone, inc_window, run_stone, run_window, n_stones):
    return values.new_empty((n_stones, values.shape[1]), dtype=torch.float32)


def _fake_class_row_sum(weight, gather, runs, n_dest, run_len):
    return weight.new_empty((n_dest, weight.shape[1]), dtype=torch.float32)


def _fake_incidence_row_sum(values, gather, runs, rev_gather, rev_runs, n_dest, run_len, rev_run_len):
    return values.new_empty((n_dest, values.shape[1]), dtype=torch.float32)


def _fake_action_row_encode(pre_w, table, edge_window, edge_class, edge_cell, edge_rev, n_cells):
    return pre_w.new_empty((n_cells, pre_w.shape[1]), dtype=torch.float32)


def _fake_cell_pass(x, emb, cell_ptr, edge_window, edge_class, win_ptr, edge_wcell, cls_ptr, edge_ccell):
    return torch.empty_like(x)


def _fake_window_latent_layout(window_pos, positions):
    return window_pos.new_empty((positions + 1,), dtype=torch.long), torch.empty_like(window_pos)


_FAKES = {
    "fused_attention": _fake_fused_attention,
    "cell_attention": _fake_segment,
    "cell_attention_plain": _fake_segment,
    "window_latent_read": _fake_latent,
    "window_latent_broadcast": _fake_latent,
    "aggregate_to_windows": _fake_aggregate_to_windows,
    "aggregate_to_stones": _fake_aggregate_to_stones,
    "class_row_sum": _fake_class_row_sum,
    "incidence_row_sum": _fake_incidence_row_sum,
    "action_row_encode": _fake_action_row_encode,
    "cell_pass": _fake_cell_pass,
    "window_latent_layout": _fake_window_latent_layout,
}

_libs: dict[str, torch.library.Library] = {}


def define(namespace: str = "mantis_b200") -> list[str]:
    """Define every op of the plug-in in ``namespace`` (reference names,
    argument lists and output contracts) with this library's CUDA kernels
    and fake implementations. Returns the qualified op names. Idempotent."""
    names = [f"{namespace}::{n}" for n in _SCHEMAS]
    if namespace in _libs:
        return names
    lib = torch.library.Library(namespace, "FRAGMENT")
    for name, schema in _SCHEMAS.items():
        lib.define(name + schema)
        lib.impl(name, _KERNELS[name], "CUDA")
        torch.library.register_fake(f"{namespace}::{name}", _FAKES[name], lib=lib)
        if name in _AUTOGRAD:
            torch.library.register_autograd(f"{namespace}::{name}", _AUTOGRAD[name], setup_context=_save_all,
                                            lib=lib)
    _libs[namespace] = lib
    return names


def install_into_reference(namespace: str = "mantisnet") -> list[str]:
    """Register this library's kernels as the CUDA implementation of each of
    the reference's ops that is defined (import the reference package
    first). Returns the ops it took over."""
    taken = []
    for name, fn in list(_KERNELS.items()) + list(_BACKWARD_KERNELS.items()):
        qual = f"{namespace}::{name}"
        try:
            torch._C._dispatch_find_schema_or_throw(qual, "")
        except RuntimeError:
            continue
        torch.library.register_kernel(qual, "cuda", fn)
        taken.append(qual)
    return taken


# ------------------------------------------------------------ backward
# The reference's backward ops (same argument lists), on this library's
# deterministic backward kernels.
def _fused_attention_backward(q, k, v, seq_lens, out, lse, grad_out):
    if lse.numel() == 0:  # a forward that kept no log-sum-exp: recompute it
        _, lse = ops.fused_attention(q, k, v, seq_lens, with_lse=True)
    return ops.stone_attention_backward(q, k, v, seq_lens, out, lse, grad_out)


def _cell_attention_backward(q, k, v, bias, vcls, seg_ptr, src, cls, qid, sseg_ptr, sqid, scls, cptr, cedge_q, m,
                             l, grad_out):
    return ops.segment_attention_backward(q, k, v, bias, vcls, seg_ptr, src, cls, m, l, grad_out, qid=qid)


def _cell_attention_plain_backward(q, k, v, bias, seg_ptr, src, cls, qid, sseg_ptr, sqid, scls, cptr, cedge_q, m,
                                   l, grad_out):
    return ops.segment_attention_backward(q, k, v, bias, None, seg_ptr, src, cls, m, l, grad_out, qid=qid)[:4]


def _window_latent_read_backward(q, k, v, window_pos, offsets, order, out, m, l, grad_out):
    return ops.window_latent_read_backward(q, k, v, offsets, order, window_pos, out, m, l, grad_out)


def _window_latent_broadcast_backward(q, k, v, window_pos, offsets, order, m, l, grad_out):
    return ops.window_latent_broadcast_backward(q, k, v, offsets, order, window_pos, m, l, grad_out)


_BACKWARD_KERNELS = {
    "fused_attention_backward": _fused_attention_backward,
    "cell_attention_backward": _cell_attention_backward,
    "cell_attention_plain_backward": _cell_attention_plain_backward,
    "window_latent_read_backward": _window_latent_read_backward,
    "window_latent_broadcast_backward": _window_latent_broadcast_backward,
}


# Autograd of the ops :func:`define` creates: save what the backward reads,
# return one gradient per input (None for index tensors and ints).
def _save_all(ctx, inputs, output):
    outs = output if isinstance(output, tuple) else (output,)
    ctx.save_for_backward(*[x for x in inputs if isinstance(x, torch.Tensor)],
                          *[o for o in outs if isinstance(o, torch.Tensor)])
    ctx.n_in = sum(isinstance(x, torch.Tensor) for x in inputs)
    ctx.ints = [x for x in inputs if not isinstance(x, torch.Tensor)]


def _bw_fused_attention(ctx, g_out, g_lse):
    q, k, v, seq_lens, out, lse = ctx.saved_tensors
    return (*_fused_attention_backward(q, k, v, seq_lens, out, lse, g_out), None)


def _bw_cell_attention(ctx, g_out, g_m, g_l):
    t = ctx.saved_tensors
    q, k, v, bias, vcls, seg_ptr, src, cls, qid = t[:9]
    m, l = t[15], t[16]
    return (*ops.segment_attention_backward(q, k, v, bias, vcls, seg_ptr, src, cls, m, l, g_out, qid=qid),
            *([None] * 9))


def _bw_cell_attention_plain(ctx, g_out, g_m, g_l):
    t = ctx.saved_tensors
    q, k, v, bias, seg_ptr, src, cls, qid = t[:8]
    m, l = t[14], t[15]
    return (*ops.segment_attention_backward(q, k, v, bias, None, seg_ptr, src, cls, m, l, g_out, qid=qid)[:4],
            *([None] * 9))


def _bw_window_latent_read(ctx, g_out, g_m, g_l):
    q, k, v, window_pos, offsets, order, out, m, l = ctx.saved_tensors
    return (*ops.window_latent_read_backward(q, k, v, offsets, order, window_pos, out, m, l, g_out), None, None,
            None)


def _bw_window_latent_broadcast(ctx, g_out, g_m, g_l):
    q, k, v, window_pos, offsets, order, out, m, l = ctx.saved_tensors
    return (*ops.window_latent_broadcast_backward(q, k, v, offsets, order, window_pos, m, l, g_out), None, None,
            None)


def _bw_action_row_encode(ctx, g_out):
    pre_w, table, edge_window, edge_class, edge_cell, edge_rev, out = ctx.saved_tensors
    gp, gt = ops.encode_rows_backward(pre_w, table, edge_window, edge_class, edge_cell, g_out)
    return gp, gt, None, None, None, None, None


_AUTOGRAD = {
    "fused_attention": _bw_fused_attention,
    "cell_attention": _bw_cell_attention,
    "cell_attention_plain": _bw_cell_attention_plain,
    "window_latent_read": _bw_window_latent_read,
    "window_latent_broadcast": _bw_window_latent_broadcast,
    "action_row_encode": _bw_action_row_encode,
}
