"""MantisNet on the B200 kernels: same module tree, parameter names, init
order and forward contract as the reference (python/mantisnet/mantisnet/
model.py), so its checkpoints load unchanged and a seeded construction draws
the same weights.

The forward is inference-only (KLENT's evaluator path). It runs on CUDA only;
every data-dependent step (CSR views, gathers, attention, reductions, norms,
composition) is a kernel of libmantis_b200.so. The dense projections follow
``Engine``'s ``gemm`` mode: by default (``tcgen05-ln``) every projection that
feeds a residual update is one fused tcgen05 launch of the library that also
writes the updated residual and the next LayerNorms; ``native`` is the
library's CUDA-core fp32 GEMM (the fp32 parity mode); ``cublas`` runs the
projections through torch (see ``Engine.__init__`` for every mode).

Numerics follow the reference's bf16 autocast contract (klent/train.py:
105-118): fp32 residual streams, LayerNorm statistics in fp32, projections in
bf16 with fp32 accumulation, every attention/softmax/segment sum in fp32,
the categorical composition in fp32. ``dtype=torch.float32`` runs every
stage in fp32 (the parity mode).
"""

from __future__ import annotations

import contextlib
import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from . import ops
from .builder import Batch
from .config import MantisConfig
from .vocab import (
    ACTION_EMPTY_CLASSES,
    COVERAGE_BUCKET_OF,
    COVERAGE_BUCKETS,
    NEAREST_BUCKETS,
    RADIUS_CLASSES,
    ADJACENCY_CLASSES,
    TACTICAL_FEATURES,
    TERN_PATTERN_CLASS_COUNTS,
    TERN_POST1_CLASSES,
)

CRITIC_LOGITS = 3
GLOBAL_ROWS = 4


@dataclass
class ModelOutput:
    """model.py:114-123."""

    policy_logits: Tensor
    q_score: Tensor
    q_values: Tensor
    value: Tensor
    value_dist: Tensor
    value_logits: Tensor


def return_mass(critic_logits: Tensor) -> tuple[Tensor, Tensor]:
    """model.py:177-186 (fp32 softmax of the three outcome logits)."""
    p = critic_logits.float().softmax(dim=-1)
    return p[..., 0], p[..., 1]


def compose_q(critic_logits: Tensor) -> Tensor:
    """model.py:189-200: Q = p_pos - p_neg, fp32 (CUDA kernel)."""
    offsets = torch.tensor([0, critic_logits.shape[0]], device=critic_logits.device)
    return ops.compose(critic_logits.reshape(-1, 3), offsets, 0.0)[1]


def compose_acting_q(critic_logits: Tensor, offsets: Tensor, mass_floor: float) -> Tensor:
    """model.py:203-220: Q over the position's floored maximum committed mass."""
    return ops.compose(critic_logits.reshape(-1, 3), offsets, mass_floor)[0]


def _mlp(d_in: int, d_hidden: int, d_out: int) -> nn.Sequential:
    return nn.Sequential(nn.Linear(d_in, d_hidden), nn.ReLU(), nn.Linear(d_hidden, d_out))


class _PairMlp(nn.Module):
    """MLP([a; b]) as lin_a(a) + lin_b(b) (model.py:246-260)."""

    def __init__(self, h: int, d_hidden: int, d_out: int) -> None:
        super().__init__()
        self.lin_a = nn.Linear(h, d_hidden)
        self.lin_b = nn.Linear(h, d_hidden, bias=False)
        self.out = nn.Linear(d_hidden, d_out)


class _Block(nn.Module):
    """One trunk block's parameters (model.py:263-369), same names and order."""

    def __init__(self, cfg: MantisConfig) -> None:
        super().__init__()
        h = cfg.h
        self.cfg = cfg
        self.ln_ws_s = nn.LayerNorm(h)
        self.ln_ws_w = nn.LayerNorm(h)
        self.u = nn.Linear(h, h, bias=False)
        self.e_ws = nn.Embedding(cfg.occ_classes, h)
        self.mlp_w = _PairMlp(h, h, h)
        if cfg.uses_cell_state:
            self.ln_cr_c = nn.LayerNorm(h)
            self.ln_cr_w = nn.LayerNorm(h)
            self.cr_wq = nn.Linear(h, h)
            self.cr_wk = nn.Linear(h, h, bias=False)
            self.cr_wv = nn.Linear(h, h)
            self.cr_wo = nn.Linear(h, h)
            self.cr_bias = nn.Parameter(torch.zeros(cfg.heads, cfg.dec_classes))
            self.cr_vclass = nn.Embedding(cfg.dec_classes, h)
            self.ln_wr_w = nn.LayerNorm(h)
            self.ln_wr_c = nn.LayerNorm(h)
            self.wr_wq = nn.Linear(h, h)
            self.wr_wk = nn.Linear(h, h, bias=False)
            self.wr_wv = nn.Linear(h, h)
            self.wr_wo = nn.Linear(h, h)
            self.wr_bias = nn.Parameter(torch.zeros(cfg.heads, cfg.dec_classes))
            if cfg.cell_nodes:
                self.ln_radius_c = nn.LayerNorm(h)
                self.ln_radius_s = nn.LayerNorm(h)
                self.radius_wq = nn.Linear(h, h)
                self.radius_wk = nn.Linear(h, h, bias=False)
                self.radius_wv = nn.Linear(h, h)
                self.radius_wo = nn.Linear(h, h)
                self.radius_bias = nn.Parameter(torch.zeros(cfg.heads, RADIUS_CLASSES))
                self.radius_vclass = nn.Embedding(RADIUS_CLASSES, h)
            if cfg.cell_adjacency:
                self.ln_adj_q = nn.LayerNorm(h)
                self.ln_adj_k = nn.LayerNorm(h)
                self.adj_wq = nn.Linear(h, h)
                self.adj_wk = nn.Linear(h, h, bias=False)
                self.adj_wv = nn.Linear(h, h)
                self.adj_wo = nn.Linear(h, h)
                self.adj_bias = nn.Parameter(torch.zeros(cfg.heads, ADJACENCY_CLASSES))
                self.adj_vclass = nn.Embedding(ADJACENCY_CLASSES, h)
            if cfg.cell_structure:
                self.ln_c = nn.LayerNorm(h)
                self.mlp_c = _PairMlp(h, h, h)
        else:
            self.ln_cp_in = nn.LayerNorm(h)
            self.u_cp = nn.Linear(h, h, bias=False)
            self.e_cp = nn.Embedding(cfg.dec_classes, h)
            self.ln_cp_w = nn.LayerNorm(h)
            self.mlp_cp = _PairMlp(h, h, h)
        self.latent_ln_read_q = nn.LayerNorm(h)
        self.latent_ln_read_w = nn.LayerNorm(h)
        self.latent_wq_read = nn.Linear(h, h)
        self.latent_wk_read = nn.Linear(h, h, bias=False)
        self.latent_wv_read = nn.Linear(h, h)
        self.latent_wo_read = nn.Linear(h, h)
        self.latent_ln_mix = nn.LayerNorm(h)
        self.latent_wq_mix = nn.Linear(h, h)
        self.latent_wk_mix = nn.Linear(h, h, bias=False)
        self.latent_wv_mix = nn.Linear(h, h)
        self.latent_wo_mix = nn.Linear(h, h)
        self.latent_ln_bcast_q = nn.LayerNorm(h)
        self.latent_ln_bcast_l = nn.LayerNorm(h)
        self.latent_wq_bcast = nn.Linear(h, h)
        self.latent_wk_bcast = nn.Linear(h, h, bias=False)
        self.latent_wv_bcast = nn.Linear(h, h)
        self.latent_wo_bcast = nn.Linear(h, h)
        self.ln_sw_w = nn.LayerNorm(h)
        self.ln_sw_s = nn.LayerNorm(h)
        self.v = nn.Linear(h, h, bias=False)
        self.e_sw = nn.Embedding(cfg.occ_classes, h)
        self.mlp_s = _PairMlp(h, h, h)
        self.ln_attn = nn.LayerNorm(h)
        self.wq = nn.Linear(h, h)
        self.wk = nn.Linear(h, h, bias=False)
        self.wv = nn.Linear(h, h)
        self.wo = nn.Linear(h, h)
        self.ln_ffn = nn.LayerNorm(h)
        self.ffn = nn.Sequential(nn.Linear(h, cfg.ffn_factor * h), nn.ReLU(), nn.Linear(cfg.ffn_factor * h, h))
        self.drop = nn.Dropout(cfg.dropout)


class MantisNet(nn.Module):
    """Embeddings, B trunk blocks, policy / action-value / state-value heads
    (model.py:695-1200). Construction order and init match the reference."""

    def __init__(self, cfg: MantisConfig | None = None) -> None:
        super().__init__()
        cfg = cfg or MantisConfig()
        self.cfg = cfg
        h = cfg.h
        self.stone_table = nn.Embedding(2, h)
        self.window_table = nn.Embedding(cfg.window_vocab, h)
        self.latent_base = nn.Parameter(torch.empty(4, h))
        self.token_moves = nn.Embedding(2, h)
        if cfg.uses_cell_state:
            self.cell_base = nn.Parameter(torch.empty(h))
        if cfg.cell_nodes or cfg.cell_structure:
            self.cell_nearest_table = nn.Embedding(NEAREST_BUCKETS, h)
        if cfg.cell_structure:
            self.cell_class_table = nn.Embedding(cfg.dec_classes, h)
            self.cell_coverage_table = nn.Embedding(COVERAGE_BUCKETS, h)
            self.register_buffer("coverage_bucket", torch.from_numpy(COVERAGE_BUCKET_OF.copy()), persistent=False)
        self.blocks = nn.ModuleList(_Block(cfg) for _ in range(cfg.blocks))
        self.register_buffer("pattern_counts", torch.from_numpy(TERN_PATTERN_CLASS_COUNTS.copy()), persistent=False)
        self.ln_out = nn.LayerNorm(h)
        self.p = nn.Linear(h, h, bias=False)
        self.e_pw = nn.Embedding(cfg.dec_classes, h)
        self.mlp_p = _PairMlp(h, cfg.policy_hidden, 1)
        self.q = nn.Linear(h, h, bias=False)
        self.e_qw = nn.Embedding(cfg.dec_classes, h)
        self.mlp_q = _PairMlp(h, cfg.policy_hidden, CRITIC_LOGITS)
        self.act_proj = nn.Linear(h, h)
        self.act_table = nn.Embedding(TERN_POST1_CLASSES, h)
        self.act_empty_base = nn.Parameter(torch.empty(h))
        self.p_act = nn.Linear(h, h, bias=False)
        self.q_act = nn.Linear(h, h, bias=False)
        self.register_buffer("act_empty_classes", torch.tensor(ACTION_EMPTY_CLASSES, dtype=torch.long),
                             persistent=False)
        if cfg.action_tactical:
            self.tactical_a = nn.Linear(TACTICAL_FEATURES, h)
            self.tactical_out = nn.Linear(h, h)
        self.value_queries = nn.Parameter(torch.empty(cfg.value_queries, h))
        self.ln_value = nn.LayerNorm(h)
        self.mlp_v = _mlp(cfg.value_queries * h, cfg.value_hidden, cfg.value_bins)
        self.register_buffer("bin_centers", torch.linspace(-1.0, 1.0, cfg.value_bins), persistent=False)
        self._init_weights()
        self._engines: dict = {}

    def _init_weights(self) -> None:
        """model.py:785-811."""
        for m in self.modules():
            if isinstance(m, nn.Embedding):
                nn.init.normal_(m.weight, std=0.02)
        nn.init.normal_(self.latent_base, std=0.02)
        if self.cfg.uses_cell_state:
            nn.init.normal_(self.cell_base, std=0.02)
        nn.init.normal_(self.value_queries, std=0.02)
        nn.init.normal_(self.act_empty_base, std=0.02)
        for head in (self.mlp_p, self.mlp_q):
            nn.init.zeros_(head.out.weight)
            nn.init.zeros_(head.out.bias)
        if self.cfg.action_tactical:
            nn.init.zeros_(self.tactical_out.weight)
            nn.init.zeros_(self.tactical_out.bias)
        if self.cfg.cell_structure:
            nn.init.zeros_(self.cell_class_table.weight)
            nn.init.zeros_(self.cell_coverage_table.weight)
            for block in self.blocks:
                nn.init.zeros_(block.mlp_c.out.weight)
                nn.init.zeros_(block.mlp_c.out.bias)

    # --------------------------------------------------------------- engine
    def engine(self, dtype: torch.dtype = torch.bfloat16, gemm: str = "tcgen05-ln") -> "Engine":
        """The prepared-weight runner for the module's device and ``dtype``;
        rebuilt when any parameter changes (in-place updates bump versions)."""
        if self.training and self.cfg.dropout > 0:
            raise NotImplementedError("the B200 forward is inference-only; call .eval() first")
        dev = next(self.parameters()).device
        if dev.type != "cuda":
            raise RuntimeError("the B200 MantisNet forward runs on CUDA only; move the module to a GPU")
        stamp = tuple((p.data_ptr(), p._version) for p in self.parameters())
        key = (dev, dtype, gemm)
        eng = self._engines.get(key)
        if eng is None or eng.stamp != stamp:
            eng = Engine(self, dtype, gemm)
            eng.stamp = stamp
            self._engines[key] = eng
        return eng

    @torch.no_grad()
    def trunk(self, batch: Batch, dtype: torch.dtype = torch.bfloat16):
        """(ln_out(w), mean latent row, cells or None) — model.py:898-985."""
        return self.engine(dtype).trunk(batch)

    @torch.no_grad()
    def cell_head_logits(self, w, g, cells, batch: Batch, dtype: torch.dtype = torch.bfloat16):
        """(policy (N,), critic (N, 3)) — model.py:1111-1139."""
        return self.engine(dtype).heads(w, g, cells, batch)

    @torch.no_grad()
    def cell_heads(self, w, g, cells, batch: Batch, mass_floor: float, dtype: torch.dtype = torch.bfloat16):
        policy, critic = self.cell_head_logits(w, g, cells, batch, dtype)
        q_score, q_values = ops.compose(critic, batch.legal_offsets, mass_floor)
        return policy, q_score, q_values

    @torch.no_grad()
    def value_head(self, w, g, batch: Batch):
        return self.engine(torch.float32).value_head(w, g, batch)

    @torch.no_grad()
    def forward(self, batch: Batch, mass_floor: float, dtype: torch.dtype = torch.bfloat16) -> ModelOutput:
        """Every head (model.py:1185-1200)."""
        eng = self.engine(dtype)
        w, g, cells = eng.trunk(batch)
        value, dist, logits = eng.value_head(w, g, batch)
        policy, critic = eng.heads(w, g, cells, batch)
        q_score, q_values = ops.compose(critic, batch.legal_offsets, mass_floor)
        return ModelOutput(policy.float(), q_score, q_values, value, dist, logits)


# ====================================================================== engine

def _f32(t: Tensor) -> Tensor:
    return t.detach().float().contiguous()


class _Lin:
    """A prepared projection: weight in the compute dtype, bias fp32 (or in
    the compute dtype for cuBLAS epilogues). In bf16 mode a weight with a
    multiple of 128 outputs also carries the swizzled image of the tcgen05
    row GEMM (``img``, K = 256 or 512), or for K a multiple of 512 one image
    per 512-column slice of K (``kparts``, summed by successive residual
    launches)."""

    __slots__ = ("w", "b", "b_cd", "n", "k", "img", "kparts")

    def __init__(self, w: Tensor, b: Tensor | None, cd: torch.dtype):
        self.w = w.detach().to(cd).contiguous()
        self.b = _f32(b) if b is not None else None
        self.b_cd = self.b.to(cd) if b is not None else None
        self.n, self.k = self.w.shape
        self.img = self.kparts = None
        if cd == torch.bfloat16 and self.w.is_cuda and self.n % 128 == 0:
            if self.k in ops.GEMM_KS:
                self.img = ops.weight_image(self.w)
            elif self.k % 512 == 0:
                self.kparts = [ops.weight_image(self.w[:, j:j + 512]) for j in range(0, self.k, 512)]


def _cat_lin(parts, cd) -> _Lin:
    """Stack linears that read the same input: rows of W, biases (zeros for
    bias-free members)."""
    ws = [l.weight for l in parts]
    bs = [l.bias if l.bias is not None else torch.zeros(l.weight.shape[0], device=l.weight.device) for l in parts]
    return _Lin(torch.cat(ws, 0), torch.cat(bs, 0), cd)


def _pair_lin(m: _PairMlp, cd) -> tuple[_Lin, _Lin]:
    """_PairMlp as one GEMM over [a | b] then the output layer."""
    return _Lin(torch.cat([m.lin_a.weight, m.lin_b.weight], 1), m.lin_a.bias, cd), _Lin(m.out.weight, m.out.bias, cd)


class _LN:
    __slots__ = ("g", "b")

    def __init__(self, ln: nn.LayerNorm):
        self.g, self.b = _f32(ln.weight), _f32(ln.bias)


class _Tables:
    """Per-batch device-side index views, derived once per forward and shared
    by every block (the reference recomputes them in the trunk prologue,
    model.py:914-936)."""

    def __init__(self, cfg: MantisConfig, b: Batch, cd: torch.dtype = torch.bfloat16):
        dev = b.stone_own.device
        self.P = int(b.attn_valid.shape[0])
        self.N_s = int(b.stone_own.shape[0])
        self.N_w = int(b.window_feat.shape[0])
        self.N_c = int(b.cell_pos.shape[0])
        self.max_t = int(b.attn_valid.shape[1])
        seq = b.attn_valid.sum(1)
        zero = torch.zeros(1, dtype=torch.long, device=dev)
        self.stone_off = torch.cat([zero, torch.cumsum(seq - GLOBAL_ROWS, 0)])
        self.tok_off = torch.cat([zero, torch.cumsum(seq, 0)])
        self.N_tok = self.N_s + GLOBAL_ROWS * self.P
        # incidence: window-major as built; stone-major by a stable sort
        self.window_ptr = ops.csr(b.inc_window, self.N_w)
        run_stone, order = ops.argsort(b.inc_stone, self.N_s)
        self.run_window = ops.gather_i64(b.inc_window, order)
        self.run_class = ops.gather_i64(b.inc_class, order)
        self.stone_ptr = ops.csr(run_stone, self.N_s)
        # window-latent layout
        self.window_pos = ops.div_i64(b.window_slot, int(b.value_valid.shape[1]))
        wp_sorted, self.wl_order = ops.argsort(self.window_pos, self.P)
        self.wl_off = ops.csr(wp_sorted, self.P)
        # decoder incidence, cell-major
        dc_sorted, dorder = ops.argsort(b.dec_cell, self.N_c)
        self.dec_window = ops.gather_i64(b.dec_window, dorder)
        self.dec_class = ops.gather_i64(b.dec_class, dorder)
        self.act_class = ops.gather_i64(b.act_class, dorder)
        self.cell_ptr = ops.csr(dc_sorted, self.N_c)
        if cfg.uses_cell_state:
            w_sorted, worder = ops.argsort(self.dec_window, self.N_w)
            self.win_ptr = ops.csr(w_sorted, self.N_w)
            self.edge_wcell = ops.gather_i64(dc_sorted, worder)
            self.edge_wclass = ops.gather_i64(self.dec_class, worder)
        # The two incidence reads (cells <- windows, windows <- cells) on the
        # block-diagonal read kernel: packed edges, each position's rows by
        # edge count and the slot tables, shared by every block.
        self.cr_slots = self.wr_slots = None
        if cfg.uses_cell_state and ops.radius_supported(cfg.heads, cfg.h, cd):
            self.pos_cell_off = ops.csr(b.cell_pos, self.P)  # cells are laid out position by position
            self.cr_order, self.cr_slots, self.cr_pack = self._read_plan(
                self.dec_window, self.dec_class, self.cell_ptr, self.pos_cell_off, self.wl_off, self.N_w,
                b.cell_pos, cfg.dec_classes)
            self.wr_order, self.wr_slots, self.wr_pack = self._read_plan(
                self.edge_wcell, self.edge_wclass, self.win_ptr, self.wl_off, self.pos_cell_off, self.N_c,
                self.window_pos, cfg.dec_classes)
        if cfg.cell_nodes:
            r_sorted, rorder = ops.argsort(b.radius_dst, self.N_c)
            self.r_src = ops.gather_i64(b.radius_src, rorder)
            self.r_cls = ops.radius_class(b.radius_orbit, b.radius_own, b.radius_on_axis, rorder)
            self.r_ptr = ops.csr(r_sorted, self.N_c)
            self.cell_off = ops.csr(b.cell_pos, self.P)  # cells are laid out position by position
            self.skip = self.cell_ptr if cfg.cell_node_scope == "uncovered" else None
            self.r_pack = self.r_order = self.r_slots = self.r_pack_slots = None
            if ops.radius_supported(cfg.heads, cfg.h, cd):
                # shared by every block's radius read: packed edges, and each
                # position's cells ordered by edge count
                self.r_pack = ops.radius_pack(self.r_src, self.r_cls, self.r_ptr, self.cell_off, self.stone_off,
                                              self.N_s, RADIUS_CLASSES)
                deg = (self.r_ptr[1:] - self.r_ptr[:-1]).clamp(max=63)
                if self.skip is not None:
                    deg = deg * (self.skip[1:] == self.skip[:-1])
                _, self.r_order = ops.argsort(b.cell_pos * 64 + deg, self.P * 64)
                self.r_slots, self.r_pack_slots = ops.radius_slots(self.r_pack, self.r_ptr, self.cell_off, self.r_order,
                                                                   self.skip)
        if cfg.cell_adjacency:
            a_sorted, aorder = ops.argsort(b.adjacency_dst, self.N_c)
            self.a_src = ops.gather_i64(b.adjacency_src, aorder)
            self.a_cls = torch.zeros_like(self.a_src)
            self.a_ptr = ops.csr(a_sorted, self.N_c)


    def _read_plan(self, src, cls, seg_ptr, q_off, s_off, n_src, q_pos, n_cls):
        """(order, slots, slot-ordered packed edges) of a block-diagonal read:
        rows of a position by ascending edge count."""
        packed = ops.radius_pack(src, cls, seg_ptr, q_off, s_off, n_src, n_cls)
        deg = (seg_ptr[1:] - seg_ptr[:-1]).clamp(max=63)
        _, order = ops.argsort(q_pos * 64 + deg, self.P * 64)
        slots, packed_slots = ops.radius_slots(packed, seg_ptr, q_off, order)
        return order, slots, packed_slots


class Engine:
    """Prepared weights plus the forward schedule over the kernels."""

    GEMM_MODES = ("tcgen05-ln", "cublas", "native")

    def __init__(self, model: MantisNet, dtype: torch.dtype, gemm: str = "tcgen05-ln"):
        """``gemm`` picks the dense-projection path:

        - ``tcgen05-ln`` (the default): every projection is a kernel of the
          library. In bf16 they run on the tcgen05 row GEMM: LayerNorm
          prologues fused where a LayerNorm feeds the projection, the
          projections that feed a residual update emit the update and the
          next LayerNorms from the same launch, and each decoder head's last
          two layers are one launch. In fp32 (the parity mode, which tensor
          -core formats cannot meet at 1e-4) they run on the CUDA-core fp32
          GEMM.
        - ``native``: the CUDA-core fp32-accumulating GEMM for every
          projection, with separate LayerNorm and residual kernels.
        - ``cublas``: the projections through torch (cuBLAS), with separate
          LayerNorm and residual kernels; a comparison path only."""
        if dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("dtype must be torch.float32 or torch.bfloat16")
        gemm = {"torch": "cublas", "tcgen05": "tcgen05-ln"}.get(gemm, gemm)
        if gemm not in self.GEMM_MODES:
            raise ValueError(f"gemm must be one of {self.GEMM_MODES}")
        self.cfg = cfg = model.cfg
        self.cd = cd = dtype
        self.gemm = gemm
        self.stamp = None
        # Optional launch timing: when a dict, the named stages of each forward
        # append a (start, end) CUDA event pair recorded on the launching stream.
        self.probe = None
        # Most sources a radius-read group stages in shared memory (None: the
        # batch's largest stone count, so every group is staged); groups of
        # more stones read their K/V rows from global memory.
        self.radius_stage_rows = None
        h = cfg.h
        m = model
        dev = m.latent_base.device
        with torch.no_grad():
            self.stone_table = _f32(m.stone_table.weight)
            self.window_table = _f32(m.window_table.weight)
            self.latent_base = _f32(m.latent_base)
            self.token_moves = _f32(m.token_moves.weight)
            if cfg.uses_cell_state:
                self.cell_base = _f32(m.cell_base)
            if cfg.cell_nodes or cfg.cell_structure:
                self.nearest_table = _f32(m.cell_nearest_table.weight)
            if cfg.cell_structure:
                self.cell_class_table = _f32(m.cell_class_table.weight)
                self.coverage_table = _f32(m.cell_coverage_table.weight)
                self.coverage_bucket = m.coverage_bucket.to(dev)
            pc = m.pattern_counts.to(dev).float()
            # §5.1 class terms of every block: counts @ [e_ws...] once, a
            # weight-only table (model.py:941-948)
            self.ws_table = (pc @ torch.cat([b.e_ws.weight.float() for b in m.blocks], 1)).contiguous() \
                if len(m.blocks) else None
            self.sw_tables = torch.cat([b.e_sw.weight.float() for b in m.blocks], 1).contiguous() \
                if len(m.blocks) else None
            self.blocks = [self._prep_block(b) for b in m.blocks]
            self.ln_out = _LN(m.ln_out)
            self.act_proj = _Lin(m.act_proj.weight, m.act_proj.bias, cd)
            self.act_table = _f32(m.act_table.weight)
            self.act_empty_base = _f32(m.act_empty_base)
            self.act_empty_classes = m.act_empty_classes.to(dev)
            # both heads' decoder matrices in one GEMM over [rows | acts]
            top = torch.cat([m.p.weight, m.p_act.weight], 1)
            bot = torch.cat([m.q.weight, m.q_act.weight], 1)
            self.dec_pq = _Lin(torch.cat([top, bot], 0), None, cd)
            self.e_pq = torch.cat([m.e_pw.weight, m.e_qw.weight], 1).float().contiguous()
            self.lin_b_pq = _Lin(torch.cat([m.mlp_p.lin_b.weight, m.mlp_q.lin_b.weight], 0), None, cd)
            self.p_lin_a = _Lin(m.mlp_p.lin_a.weight, m.mlp_p.lin_a.bias, cd)
            self.q_lin_a = _Lin(m.mlp_q.lin_a.weight, m.mlp_q.lin_a.bias, cd)
            self.p_out = _Lin(m.mlp_p.out.weight, m.mlp_p.out.bias, cd)
            self.q_out = _Lin(m.mlp_q.out.weight, m.mlp_q.out.bias, cd)
            # fp32 output layers for the fused head launch
            self.head_out32 = [(_f32(m.mlp_p.out.weight), _f32(m.mlp_p.out.bias)),
                               (_f32(m.mlp_q.out.weight), _f32(m.mlp_q.out.bias))]
            if cfg.action_tactical:
                self.tactical_a = _Lin(m.tactical_a.weight, m.tactical_a.bias, cd)
                self.tactical_out = _Lin(m.tactical_out.weight, m.tactical_out.bias, cd)
            self.value_queries = _f32(m.value_queries)
            self.ln_value = _LN(m.ln_value)
            self.mlp_v0 = (_f32(m.mlp_v[0].weight), _f32(m.mlp_v[0].bias))
            self.mlp_v2 = (_f32(m.mlp_v[2].weight), _f32(m.mlp_v[2].bias))
            self.bin_centers = m.bin_centers.to(dev).float()
        self.h = h

    def _prep_block(self, b: _Block) -> dict:
        cfg, cd = self.cfg, self.cd
        d = {
            "ln_ws_s": _LN(b.ln_ws_s), "ln_ws_w": _LN(b.ln_ws_w), "u": _Lin(b.u.weight, None, cd),
            "mlp_w": _pair_lin(b.mlp_w, cd),
            "ln_sw_w": _LN(b.ln_sw_w), "ln_sw_s": _LN(b.ln_sw_s), "v": _Lin(b.v.weight, None, cd),
            "mlp_s": _pair_lin(b.mlp_s, cd),
            "ln_attn": _LN(b.ln_attn), "qkv": _cat_lin([b.wq, b.wk, b.wv], cd), "wo": _Lin(b.wo.weight, b.wo.bias, cd),
            "ln_ffn": _LN(b.ln_ffn), "ffn0": _Lin(b.ffn[0].weight, b.ffn[0].bias, cd),
            "ffn2": _Lin(b.ffn[2].weight, b.ffn[2].bias, cd),
            "ln_read_q": _LN(b.latent_ln_read_q), "ln_read_w": _LN(b.latent_ln_read_w),
            "wq_read": _Lin(b.latent_wq_read.weight, b.latent_wq_read.bias, cd),
            "kv_read": _cat_lin([b.latent_wk_read, b.latent_wv_read], cd),
            "wo_read": _Lin(b.latent_wo_read.weight, b.latent_wo_read.bias, cd),
            "ln_mix": _LN(b.latent_ln_mix), "qkv_mix": _cat_lin([b.latent_wq_mix, b.latent_wk_mix, b.latent_wv_mix], cd),
            "wo_mix": _Lin(b.latent_wo_mix.weight, b.latent_wo_mix.bias, cd),
            "ln_bcast_q": _LN(b.latent_ln_bcast_q), "ln_bcast_l": _LN(b.latent_ln_bcast_l),
            "wq_bcast": _Lin(b.latent_wq_bcast.weight, b.latent_wq_bcast.bias, cd),
            "kv_bcast": _cat_lin([b.latent_wk_bcast, b.latent_wv_bcast], cd),
            "wo_bcast": _Lin(b.latent_wo_bcast.weight, b.latent_wo_bcast.bias, cd),
        }
        if cfg.uses_cell_state:
            d.update({
                "ln_cr_c": _LN(b.ln_cr_c), "ln_cr_w": _LN(b.ln_cr_w),
                "cr_wq": _Lin(b.cr_wq.weight, b.cr_wq.bias, cd), "cr_kv": _cat_lin([b.cr_wk, b.cr_wv], cd),
                "cr_wo": _Lin(b.cr_wo.weight, b.cr_wo.bias, cd), "cr_bias": _f32(b.cr_bias),
                "cr_vclass": b.cr_vclass.weight.detach().to(cd).contiguous(),
                "ln_wr_w": _LN(b.ln_wr_w), "ln_wr_c": _LN(b.ln_wr_c),
                "wr_wq": _Lin(b.wr_wq.weight, b.wr_wq.bias, cd), "wr_kv": _cat_lin([b.wr_wk, b.wr_wv], cd),
                "wr_wo": _Lin(b.wr_wo.weight, b.wr_wo.bias, cd), "wr_bias": _f32(b.wr_bias),
            })
            if cfg.cell_nodes:
                d.update({
                    "ln_radius_c": _LN(b.ln_radius_c), "ln_radius_s": _LN(b.ln_radius_s),
                    "radius_wq": _Lin(b.radius_wq.weight, b.radius_wq.bias, cd),
                    "radius_kv": _cat_lin([b.radius_wk, b.radius_wv], cd),
                    "radius_wo": _Lin(b.radius_wo.weight, b.radius_wo.bias, cd),
                    "radius_bias": _f32(b.radius_bias),
                    "radius_vclass": b.radius_vclass.weight.detach().to(cd).contiguous(),
                })
            if cfg.cell_adjacency:
                d.update({
                    "ln_adj_q": _LN(b.ln_adj_q), "ln_adj_k": _LN(b.ln_adj_k),
                    "adj_wq": _Lin(b.adj_wq.weight, b.adj_wq.bias, cd), "adj_kv": _cat_lin([b.adj_wk, b.adj_wv], cd),
                    "adj_wo": _Lin(b.adj_wo.weight, b.adj_wo.bias, cd), "adj_bias": _f32(b.adj_bias),
                    "adj_vclass": b.adj_vclass.weight.detach().to(cd).contiguous(),
                })
            if cfg.cell_structure:
                d.update({"ln_c": _LN(b.ln_c), "mlp_c": _pair_lin(b.mlp_c, cd)})
        else:
            d.update({
                "ln_cp_in": _LN(b.ln_cp_in), "u_cp": _Lin(b.u_cp.weight, None, cd), "e_cp": _f32(b.e_cp.weight),
                "ln_cp_w": _LN(b.ln_cp_w), "mlp_cp": _pair_lin(b.mlp_cp, cd),
            })
        return d

    # ----------------------------------------------------------- primitives
    def _tc(self, lin: _Lin, x: Tensor) -> bool:
        """Whether act(x @ W^T) runs on the tcgen05 row GEMM."""
        return (self.gemm == "tcgen05-ln" and lin.img is not None and x.dtype == torch.bfloat16 and x.dim() == 2
                and x.stride(1) == 1 and x.shape[1] == lin.k)

    def linear(self, x: Tensor, lin: _Lin, relu: bool = False, out: Tensor | None = None,
               add: Tensor | None = None) -> Tensor:
        """act(x @ W^T + b (+ add)) in the compute dtype, fp32 accumulation;
        ``add`` is an fp32 addend of the output's shape."""
        if self._tc(lin, x):
            return ops.gemm_rows(x, lin.img, bias=lin.b, relu=relu, out=out, add=add)
        if self.gemm != "cublas":
            if add is None:
                return ops.linear_native(x, lin.w, lin.b, relu=relu, out_dtype=self.cd, out=out)
            y = ops.linear_native(x, lin.w, lin.b, out_dtype=torch.float32)
            ops.residual_add(y, add)
            if relu:
                y.relu_()
            if out is None:
                return y.to(self.cd)
            out.copy_(y)
            return out
        if lin.b_cd is None:
            y = torch.matmul(x, lin.w.t(), out=out) if out is not None else torch.matmul(x, lin.w.t())
        elif relu and add is None:
            y = torch._addmm_activation(lin.b_cd, x, lin.w.t(), use_gelu=False)
            if out is not None:
                out.copy_(y)
                y = out
        else:
            y = torch.addmm(lin.b_cd, x, lin.w.t(), out=out) if out is not None else torch.addmm(lin.b_cd, x, lin.w.t())
        if add is not None:
            y.copy_(y.float() + add)
        if relu and (lin.b_cd is None or add is not None):
            y.relu_()
        return y

    @contextlib.contextmanager
    def timed(self, name: str):
        """Bracket the launches of one stage with CUDA events when probing."""
        if self.probe is None:
            yield
            return
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        yield
        end.record()
        self.probe.setdefault(name, []).append((start, end))

    def ln(self, x: Tensor, p: _LN, out: Tensor | None = None, dtype=None) -> Tensor:
        return ops.layer_norm(x, p.g, p.b, out_dtype=dtype or self.cd, out=out)

    def ln_linear(self, x: Tensor, p: _LN, lin: _Lin, relu: bool = False) -> Tensor:
        """act(LN(x) @ W^T + b): one tcgen05 launch with the LayerNorm in the
        prologue (x fp32, width 256, any multiple of 128 outputs), else LN
        then GEMM."""
        if (self.gemm == "tcgen05-ln" and lin.img is not None and lin.k == ops.GEMM_K and x.dtype == torch.float32
                and self.cd == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1):
            return ops.gemm_rows(x, lin.img, bias=lin.b, gamma=p.g, beta=p.b, relu=relu)
        return self.linear(self.ln(x, p), lin, relu=relu)

    def linear_update(self, a: Tensor, lin: _Lin, x: Tensor, lns) -> list[Tensor]:
        """x += a @ W^T + b, then the LayerNorms ``lns`` of the updated rows
        (as ``update``): one tcgen05 launch in ``tcgen05-ln`` mode."""
        if (self._tc(lin, a) and lin.n == ops.GEMM_N and lin.k == ops.GEMM_K and 1 <= len(lns) <= 3
                and x.dtype == torch.float32 and x.stride(1) == 1
                and all(not isinstance(e, tuple) or e[1] is None or e[1].dtype == torch.bfloat16 for e in lns)):
            outs = []
            for e in lns:
                p, o = e if isinstance(e, tuple) else (e, None)
                if o is None:
                    o = torch.empty(x.shape[0], x.shape[1], dtype=self.cd, device=x.device)
                outs.append((p.g, p.b, o))
            if self.probe is not None:  # algorithmic bytes of the launch: a, residual in + out, outputs
                self.probe.setdefault("resid_ln_bytes", []).append(x.shape[0] * (512 + 2048 + 512 * len(outs)))
            with self.timed("resid_ln"):
                return ops.gemm_rows_ln(a, lin.img, lin.b, x, outs)
        return self.update(x, self.linear(a, lin), lns)

    def linear_residual(self, a: Tensor, lin: _Lin, x: Tensor) -> None:
        """x += a @ W^T + b with the residual add in the GEMM epilogue (a
        K wider than 512 is summed over 512-column slices, one launch each)."""
        if (self.gemm == "tcgen05-ln" and lin.n == ops.GEMM_N and a.dtype == torch.bfloat16 and a.stride(1) == 1
                and x.dtype == torch.float32 and x.stride(1) == 1 and a.shape[1] == lin.k):
            if lin.img is not None:
                ops.gemm_rows(a, lin.img, bias=lin.b, residual=x)
                return
            if lin.kparts is not None:
                for j, img in enumerate(lin.kparts):
                    ops.gemm_rows(a[:, j * 512:(j + 1) * 512], img, bias=lin.b if j == 0 else None, residual=x)
                return
        ops.residual_add(x, self.linear(a, lin))

    def pair_mlp_residual(self, x: Tensor, a_ln: _LN, agg_writer, mlp) -> None:
        """x += out(relu([ln(x) | agg] @ [Wa | Wb]^T + ba)) with ``agg_writer``
        filling the right half of the staging buffer."""
        h = self.h
        buf = torch.empty(x.shape[0], 2 * h, dtype=self.cd, device=x.device)
        self.ln(x, a_ln, out=buf[:, :h])
        agg_writer(buf[:, h:])
        hid = self.linear(buf, mlp[0], relu=True)
        self.linear_residual(hid, mlp[1], x)

    # ---------------------------------------------------------------- trunk
    def update(self, x: Tensor, y: Tensor | None, lns) -> list[Tensor]:
        """x += y, then one LayerNorm per ``lns`` entry, in a single pass over
        x. Entries are ``_LN`` (a new compute-dtype tensor), or ``(_LN, out)``
        with ``out`` a preallocated destination (dtype and stride taken from
        it). Returns the outputs in order."""
        outs = []
        for e in lns:
            p, o = e if isinstance(e, tuple) else (e, None)
            if o is None:
                o = torch.empty(x.shape[0], x.shape[1], dtype=self.cd, device=x.device)
            outs.append((p.g, p.b, o))
        for j in range(0, max(len(outs), 1), 3):
            ops.add_ln(x, y if j == 0 else None, outs=outs[j:j + 3])
        return [o for _, _, o in outs]

    # ---------------------------------------------------------------- trunk
    def trunk(self, b: Batch, for_heads: bool = False):
        """model.py:898-985. Every update of the large residual streams (w per
        window, c per cell) also emits the LayerNorms of the next stages that
        read them, so a stream row is read and written once per update.

        Returns ln_out(w) and cells fp32, as the reference does. With
        ``for_heads`` (the evaluate path, whose only readers are the heads'
        compute-dtype GEMMs) the final LayerNorms write compute-dtype rows
        instead, cells straight into the left half of the decoder's input
        buffer; the values are the same rows rounded where the reference's
        autocast GEMMs round them."""
        cfg, cd, h = self.cfg, self.cd, self.h
        T = _Tables(cfg, b, cd)
        self.tables = T
        dev = b.stone_own.device
        direct = for_heads and cfg.uses_cell_state and cfg.cell_nodes
        self._exit_w = torch.empty(T.N_w, h, dtype=cd if direct else torch.float32, device=dev)
        self._head_buf = self._exit_c = None
        if cfg.uses_cell_state:
            if direct:
                self._head_buf = torch.empty(T.N_c, 2 * h, dtype=cd, device=dev)
                self._exit_c = self._head_buf[:, :h]
            else:
                self._exit_c = torch.empty(T.N_c, h, dtype=torch.float32, device=dev)
        s = ops.embed(self.stone_table, b.stone_own)
        w = ops.embed(self.window_table, b.window_feat)
        slot = torch.arange(T.P * GLOBAL_ROWS, device=dev) % GLOBAL_ROWS
        g = ops.embed(self.latent_base, slot, self.token_moves, b.moves_idx.repeat_interleave(GLOBAL_ROWS))
        c = None
        if cfg.uses_cell_state:
            add = None
            if cfg.cell_structure:
                classes = ops.run_reduce(self.cell_class_table, T.dec_class, T.cell_ptr, T.N_c)
                degree = (T.cell_ptr[1:] - T.cell_ptr[:-1]).clamp(max=len(COVERAGE_BUCKET_OF) - 1)
                add = classes + self.coverage_table[self.coverage_bucket[degree]] \
                    + self.nearest_table[b.cell_nearest]
                add = add.contiguous()
            if cfg.cell_nodes:
                c = ops.cell_init(T.cell_ptr, b.cell_nearest, self.nearest_table, self.cell_base, add)
            else:
                c = self.cell_base.expand(T.N_c, h).clone()
                if add is not None:
                    c += add
        sw_all = ops.run_reduce(self.sw_tables, T.run_class, T.stone_ptr, T.N_s) if self.blocks else None
        nb = len(self.blocks)
        w_out = cells = None
        if nb:
            first = self.blocks[0]
            buf_w = torch.empty(T.N_w, 2 * h, dtype=cd, device=dev)
            self.update(w, None, [(first["ln_ws_w"], buf_w[:, :h])])
            zc = self.update(c, None, [first["ln_cr_c"]])[0] if cfg.uses_cell_state else None
            for i, blk in enumerate(self.blocks):
                nxt = self.blocks[i + 1] if i + 1 < nb else None
                s, w, g, c, buf_w, zc, w_out, cells = self._block(
                    i, blk, nxt, s, w, g, c, b, T, sw_all, buf_w, zc, update_stones=i + 1 < nb)
        else:
            w_out = self.ln(w, self.ln_out, dtype=torch.float32)
            if cfg.uses_cell_state:
                cells = self.ln(c, self.ln_out, dtype=torch.float32)
        g_ln = self.ln(g, self.ln_out, dtype=torch.float32)
        global_rows = ops.latent_mean(g_ln, T.P)
        if cfg.uses_cell_state and not cfg.cell_nodes:
            base = F.layer_norm(self.cell_base, (h,), self.ln_out.g, self.ln_out.b, 1e-5)
            covered = (T.cell_ptr[1:] > T.cell_ptr[:-1])[:, None]
            cells = torch.where(covered, cells, base)
        return w_out, global_rows, cells

    def _exit_lns(self, nxt, key):
        """The LayerNorm a stream's last update of a block feeds: the next
        block's entry norm, or the trunk's shared ln_out (fp32 output)."""
        return nxt[key] if nxt is not None else None

    def _block(self, i, blk, nxt, s, w, g, c, b, T: _Tables, sw_all, buf_w, zc, update_stones: bool):
        """model.py:543-692."""
        cfg, cd, h = self.cfg, self.cd, self.h
        # §5.1 windows <- stones (sum) + per-pattern class rows; buf_w's left
        # half already holds LN_ws_w(w)
        x = self.ln_linear(s, blk["ln_ws_s"], blk["u"])
        ops.run_reduce(x, b.inc_stone, T.window_ptr, T.N_w, add=self.ws_table[:, i * h:(i + 1) * h],
                       add_idx=b.window_feat, out=buf_w[:, h:])
        hid_w = self.linear(buf_w, blk["mlp_w"][0], relu=True)
        # §5.1b
        if cfg.uses_cell_state:
            zw_cr, zw_wr = self.linear_update(hid_w, blk["mlp_w"][1], w, [blk["ln_cr_w"], blk["ln_wr_w"]])
            back, c, zc, cells = self._cell_stage(blk, nxt, s, c, T, zc, zw_cr, zw_wr)
            zw_sw, zw_read, zw_bq = self.linear_update(back, blk["wr_wo"], w,
                                                       [blk["ln_sw_w"], blk["ln_read_w"], blk["ln_bcast_q"]])
        else:
            y = self.linear(hid_w, blk["mlp_w"][1])
            buf2 = torch.empty(T.N_w, 2 * h, dtype=cd, device=w.device)
            zin, _ = self.update(w, y, [blk["ln_cp_in"], (blk["ln_cp_w"], buf2[:, :h])])
            xr = self.linear(zin, blk["u_cp"])
            buf2[:, h:].copy_(ops.cell_pass(xr, blk["e_cp"], b.relay_cell_ptr, b.relay_window, b.relay_class,
                                            b.relay_win_ptr, b.relay_wcell, b.relay_cls_ptr, b.relay_ccell))
            y = self.linear(self.linear(buf2, blk["mlp_cp"][0], relu=True), blk["mlp_cp"][1])
            cells = None
            zw_sw, zw_read, zw_bq = self.update(w, y, [blk["ln_sw_w"], blk["ln_read_w"], blk["ln_bcast_q"]])
        # §5.2 stones <- windows (fp32 sum) + class rows
        yv = self.linear(zw_sw, blk["v"])
        sw = sw_all[:, i * h:(i + 1) * h]
        self.pair_mlp_residual(
            s, blk["ln_sw_s"],
            lambda out: ops.run_reduce(yv, T.run_window, T.stone_ptr, T.N_s, add=sw, out=out),
            blk["mlp_s"])
        # §5.3 attention over [latents; stones]
        tok = ops.tokens_gather(g, s, T.stone_off, T.tok_off, T.N_tok)
        qkv = self.ln_linear(tok, blk["ln_attn"], blk["qkv"])
        if update_stones:
            att = ops.stone_attention_ragged(qkv, T.tok_off, cfg.heads, T.max_t)
            ops.tokens_scatter_add(g, s, T.stone_off, T.tok_off, self.linear(att, blk["wo"]), update_stones=True)
        else:
            att = ops.stone_attention_ragged(qkv, T.tok_off, cfg.heads, T.max_t, max_queries=GLOBAL_ROWS,
                                             out_dtype=cd)
            self.linear_residual(att, blk["wo"], g)
        # window-latent cycle (model.py:492-541)
        q = self.ln_linear(g, blk["ln_read_q"], blk["wq_read"])
        kv = self.linear(zw_read, blk["kv_read"])
        read = ops.latent_read(q, kv[:, :h], kv[:, h:], cfg.heads, T.wl_off, T.wl_order, out_dtype=cd)
        self.linear_residual(read, blk["wo_read"], g)
        qkv = self.ln_linear(g, blk["ln_mix"], blk["qkv_mix"])
        self.linear_residual(ops.latent_mix(qkv, cfg.heads, cd), blk["wo_mix"], g)
        kv = self.ln_linear(g, blk["ln_bcast_l"], blk["kv_bcast"])
        q = self.linear(zw_bq, blk["wq_bcast"])
        bc = ops.latent_broadcast(q, kv[:, :h], kv[:, h:], cfg.heads, T.window_pos, T.P, out_dtype=cd)
        w_out = None
        if nxt is not None:
            buf_w = torch.empty(T.N_w, 2 * h, dtype=cd, device=w.device)
            self.linear_update(bc, blk["wo_bcast"], w, [(nxt["ln_ws_w"], buf_w[:, :h])])
        else:
            w_out = self._exit_w
            self.linear_update(bc, blk["wo_bcast"], w, [(self.ln_out, w_out)])
        # FFN (row-wise; the stone half is skipped in the last block)
        for x_ in ((s, g) if update_stones else (g,)):
            hid = self.ln_linear(x_, blk["ln_ffn"], blk["ffn0"], relu=True)
            self.linear_residual(hid, blk["ffn2"], x_)
        return s, w, g, c, buf_w, zc, w_out, cells

    def _cell_stage(self, blk, nxt, s, c, T: _Tables, zc_cr, zw_cr, zw_wr):
        """model.py:397-490. Returns the window read-back rows (before their
        output projection, which the caller fuses with the window update),
        the updated cells, the next block's LN_cr_c(c) and, after the last
        block, ln_out(c)."""
        cfg, cd, h = self.cfg, self.cd, self.h
        zstate = self.ln(c, blk["ln_c"]) if cfg.cell_structure else None
        q = self.linear(zc_cr, blk["cr_wq"])
        kv = self.linear(zw_cr, blk["cr_kv"])
        with self.timed("cell_read"):
            if T.cr_slots is not None:
                read = ops.radius_read(q, kv[:, :h], kv[:, h:], blk["cr_bias"], blk["cr_vclass"], T.cell_ptr,
                                       T.cr_pack, T.pos_cell_off, T.wl_off, 1, order=T.cr_order, out_dtype=cd,
                                       slots=T.cr_slots)
            else:
                read = ops.segment_attention(q, kv[:, :h], kv[:, h:], blk["cr_bias"], blk["cr_vclass"], T.cell_ptr,
                                             T.dec_window, T.dec_class, out_dtype=cd)
        simple = not (cfg.cell_structure or cfg.cell_adjacency)
        exit_ln = (nxt["ln_cr_c"], None) if nxt is not None else (self.ln_out, self._exit_c)
        reads = None
        if cfg.cell_nodes and not cfg.cell_structure:
            (zc_rad,) = self.linear_update(read, blk["cr_wo"], c, [blk["ln_radius_c"]])
        else:
            reads = self.linear(read, blk["cr_wo"])
        if cfg.cell_nodes:
            if reads is not None:
                (zc_rad,) = self.update(c, reads, [blk["ln_radius_c"]])
            q = self.linear(zc_rad, blk["radius_wq"])
            kv = self.ln_linear(s, blk["ln_radius_s"], blk["radius_kv"])
            stage = self.radius_stage_rows if self.radius_stage_rows is not None else T.max_t - GLOBAL_ROWS
            with self.timed("radius_read"):
                if T.r_pack is not None:
                    read = ops.radius_read(q, kv[:, :h], kv[:, h:], blk["radius_bias"], blk["radius_vclass"], T.r_ptr,
                                           T.r_pack_slots, T.cell_off, T.stone_off, stage, order=T.r_order,
                                           skip_ptr=T.skip, out_dtype=cd, slots=T.r_slots)
                elif ops.grouped_supported(cfg.heads, h, cd):
                    # block-diagonal: position p's cells read only position p's stones
                    read = ops.segment_attention_grouped(
                        q, kv[:, :h], kv[:, h:], blk["radius_bias"], blk["radius_vclass"], T.r_ptr, T.r_src,
                        T.r_cls, T.cell_off, T.stone_off,
                        self.radius_stage_rows if self.radius_stage_rows is not None else T.max_t - GLOBAL_ROWS,
                        skip_ptr=T.skip, out_dtype=cd)
                else:
                    read = ops.segment_attention(q, kv[:, :h], kv[:, h:], blk["radius_bias"], blk["radius_vclass"],
                                                 T.r_ptr, T.r_src, T.r_cls, skip_ptr=T.skip, out_dtype=cd)
            if simple:
                zc_wr, zc_out = self.linear_update(read, blk["radius_wo"], c, [blk["ln_wr_c"], exit_ln])
            else:
                y = self.linear(read, blk["radius_wo"])
                if cfg.cell_structure:
                    reads = (reads.float() + y.float()).to(cd)
        else:
            y = reads
        if simple and not cfg.cell_nodes:
            zc_wr, zc_out = self.update(c, y, [blk["ln_wr_c"], exit_ln])
        elif not simple:
            self.update(c, y, [])
            if cfg.cell_structure:
                mlp = blk["mlp_c"]
                buf = torch.cat([zstate, reads], 1)
                self.linear_residual(self.linear(buf, mlp[0], relu=True), mlp[1], c)
            if cfg.cell_adjacency:
                q = self.ln_linear(c, blk["ln_adj_q"], blk["adj_wq"])
                kv = self.ln_linear(c, blk["ln_adj_k"], blk["adj_kv"])
                read = ops.segment_attention(q, kv[:, :h], kv[:, h:], blk["adj_bias"], blk["adj_vclass"], T.a_ptr,
                                             T.a_src, T.a_cls, skip_ptr=T.skip, out_dtype=cd)
                self.linear_residual(read, blk["adj_wo"], c)
            zc_wr, zc_out = self.update(c, None, [blk["ln_wr_c"], exit_ln])
        q = self.linear(zw_wr, blk["wr_wq"])
        kv = self.linear(zc_wr, blk["wr_kv"])
        with self.timed("window_read"):
            if T.wr_slots is not None:
                back = ops.radius_read(q, kv[:, :h], kv[:, h:], blk["wr_bias"], None, T.win_ptr, T.wr_pack, T.wl_off,
                                       T.pos_cell_off, 1, order=T.wr_order, out_dtype=cd, slots=T.wr_slots)
            else:
                back = ops.segment_attention(q, kv[:, :h], kv[:, h:], blk["wr_bias"], None, T.win_ptr, T.edge_wcell,
                                             T.edge_wclass, out_dtype=cd)
        if nxt is not None:
            return back, c, zc_out, None
        return back, c, None, zc_out

    # ---------------------------------------------------------------- heads
    def heads(self, w: Tensor, g: Tensor, cells, b: Batch):
        """policy logits (N,) fp32 and critic logits (N, 3) — model.py:1031-1139."""
        cfg, cd, h = self.cfg, self.cd, self.h
        T = getattr(self, "tables", None)
        if T is None or T.N_c != b.cell_pos.shape[0]:
            T = _Tables(cfg, b, cd)
        n_c = T.N_c
        pre = self.linear(w.to(cd), self.act_proj)
        # decoder input [cells | action rows]; the evaluate path's trunk has
        # already written cells into the left half of its buffer
        head_buf = getattr(self, "_head_buf", None)
        in_place = (cfg.uses_cell_state and head_buf is not None and cells is not None
                    and cells.data_ptr() == head_buf.data_ptr() and head_buf.shape == (n_c, 2 * h))
        buf = head_buf if in_place else torch.empty(n_c, 2 * h, dtype=cd, device=w.device)
        enc = dict(empty_counts=b.act_empty.contiguous(), empty_base=self.act_empty_base,
                   empty_cls=self.act_empty_classes)
        if cfg.action_tactical:
            acts = ops.row_encode(pre, self.act_table, T.dec_window, T.act_class, T.cell_ptr, n_c,
                                  out_dtype=torch.float32, **enc)
            t = self.linear(b.act_tactical.to(cd), self.tactical_a, relu=True)
            self.linear_residual(t, self.tactical_out, acts)
            buf[:, h:].copy_(acts)
        else:
            ops.row_encode(pre, self.act_table, T.dec_window, T.act_class, T.cell_ptr, n_c, out=buf[:, h:], **enc)
        if not in_place:
            if cfg.uses_cell_state:
                buf[:, :h].copy_(cells)
            else:
                ops.run_reduce(w, T.dec_window, T.cell_ptr, n_c, out=buf[:, :h])
        # (N_c, 2H): [p-head | q-head] = [cells | acts] @ W_dec^T + sum of the
        # cell's decoder class rows
        extra = ops.run_reduce(self.e_pq, T.dec_class, T.cell_ptr, n_c)
        lin = self.dec_pq
        if self._tc(lin, buf) and lin.k == 512 and lin.n == 2 * h == 512:
            # K = 512 with 512 outputs: as two 256-output launches on the
            # weight-stationary plan (each image half is an image of its own)
            base = torch.empty(n_c, 2 * h, dtype=cd, device=buf.device)
            half = lin.img.view(-1).shape[0] // 2
            for j in range(2):
                img = lin.img.view(-1)[j * half:(j + 1) * half].view(h, lin.k)
                ops.gemm_rows(buf, img, bias=None if lin.b is None else lin.b[j * h:(j + 1) * h],
                              add=extra[:, j * h:(j + 1) * h], out=base[:, j * h:(j + 1) * h])
        else:
            base = self.linear(buf, lin, add=extra)
        gh = self.linear(g.to(cd), self.lin_b_pq)  # (P, 2 * P_H)
        ph = cfg.policy_hidden
        outs = []
        for j, (lin_a, out_lin) in enumerate(((self.p_lin_a, self.p_out), (self.q_lin_a, self.q_out))):
            x_j = base[:, j * h:(j + 1) * h]
            t_j = gh[:, j * ph:(j + 1) * ph]
            if self._tc(lin_a, x_j) and lin_a.n in (128, 256) and out_lin.n <= 4:
                w_out, b_out = self.head_out32[j]
                outs.append(ops.gemm_head(x_j, lin_a.img, lin_a.b, t_j, b.cell_pos, w_out, b_out))
                continue
            pre_j = self.linear(x_j, lin_a)
            ops.add_gather(pre_j, t_j.contiguous(), b.cell_pos, relu=True)
            outs.append(self.linear(pre_j, out_lin))
        return outs[0].float().reshape(-1), outs[1].float()

    def evaluate(self, b: Batch):
        """trunk + heads for the evaluator closure: (policy (N,), critic (N, 3))."""
        w, g, cells = self.trunk(b, for_heads=True)
        return self.heads(w, g, cells, b)

    def value_head(self, w: Tensor, g: Tensor, b: Batch):
        """model.py:1160-1183 (full forward only; KLENT skips it): one kernel
        per batch (ops.value_head)."""
        T = getattr(self, "tables", None)
        if T is None or T.N_w != b.window_feat.shape[0] or T.P != g.shape[0]:
            T = _Tables(self.cfg, b, self.cd)
        w = w if w.stride(1) == 1 else w.contiguous()
        return ops.value_head(g.float().contiguous(), w, T.wl_off, T.wl_order, b.window_slot, b.value_valid,
                              self.ln_value.g, self.ln_value.b, self.value_queries, self.mlp_v0[0], self.mlp_v0[1],
                              self.mlp_v2[0], self.mlp_v2[1], self.bin_centers)
