"""Model configuration (reference python/mantisnet/mantisnet/model.py:49-111)."""

from __future__ import annotations

from dataclasses import asdict, dataclass

from .vocab import TERN_DEC_CLASSES, TERN_OCC_CLASSES, TERN_PATTERNS

CELL_NODE_SCOPES = ("all", "uncovered")


@dataclass(frozen=True)
class MantisConfig:
    """Same fields, defaults and validation as the reference ``MantisConfig``."""

    h: int = 128
    blocks: int = 4
    heads: int = 4
    ffn_factor: int = 2
    value_queries: int = 4
    value_bins: int = 65
    policy_hidden: int = 128
    value_hidden: int = 128
    dropout: float = 0.0
    cell_latents: bool = False
    cell_nodes: bool = False
    cell_node_scope: str = "all"
    cell_adjacency: bool = False
    cell_structure: bool = False
    action_tactical: bool = False

    def __post_init__(self) -> None:
        if self.h % self.heads != 0:
            raise ValueError(f"H={self.h} must divide into A={self.heads} heads")
        if self.value_bins % 2 == 0:
            raise ValueError(f"K={self.value_bins} must be odd so an exact-zero bin exists")
        if self.cell_adjacency and not self.cell_nodes:
            raise ValueError("cell_adjacency requires cell_nodes=True")
        if self.cell_node_scope not in CELL_NODE_SCOPES:
            raise ValueError(f"cell_node_scope must be one of {CELL_NODE_SCOPES}, got {self.cell_node_scope!r}")
        if self.cell_node_scope != "all" and not self.cell_nodes:
            raise ValueError(f"cell_node_scope={self.cell_node_scope!r} requires cell_nodes=True")
        if self.cell_structure and not self.cell_latents:
            raise ValueError("cell_structure requires cell_latents=True")

    @property
    def uses_cell_state(self) -> bool:
        return self.cell_latents or self.cell_nodes

    @property
    def window_vocab(self) -> int:
        return TERN_PATTERNS

    @property
    def dec_classes(self) -> int:
        return TERN_DEC_CLASSES

    @property
    def occ_classes(self) -> int:
        return TERN_OCC_CLASSES

    def to_dict(self) -> dict:
        return asdict(self)
