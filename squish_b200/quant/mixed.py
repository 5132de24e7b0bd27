"""Layer-selective mixed precision: which weight format each projection gets.

The reference's MixedPrecisionRouter (squish/quant/quantizer.py:737-800): the first two and
last two decoder layers (all layers when there are fewer than four) stay INT4; elsewhere the
MLP gate/up projections go to SQINT2 and the attention projections (q, k, v, o) to INT3; every
other weight is INT4. Non-weight tensors are not routed. Every format it picks has a GEMM
code format here (SQINT2 with its input rotation), and fused groups (q/k/v, gate/up) always
receive one format, so a routed model runs without re-encoding.
"""
from __future__ import annotations

import re

_LAYER = re.compile(r"\.layers\.(\d+)\.")
_PROJ = re.compile(r"\.(?P<proj>q_proj|k_proj|v_proj|o_proj|gate_proj|up_proj|down_proj)\.weight$")

FORMAT_KIND = {"int4": "q4a", "int3": "q3", "sqint2": "sqint2"}


class MixedPrecisionRouter:
    SQINT2_PROJS = frozenset({"gate_proj", "up_proj"})
    INT3_PROJS = frozenset({"q_proj", "k_proj", "v_proj", "o_proj"})

    def __init__(self, n_layers: int) -> None:
        if n_layers < 1:
            raise ValueError(f"n_layers must be >= 1, got {n_layers}")
        self.n_layers = n_layers
        self.boundary_layers = frozenset(range(n_layers)) if n_layers < 4 else \
            frozenset({0, 1, n_layers - 2, n_layers - 1})

    def format_for(self, name: str) -> str | None:
        if not name.endswith(".weight"):
            return None
        m = _LAYER.search(name)
        if m is None:
            return None
        layer = int(m.group(1))
        if layer >= self.n_layers or layer in self.boundary_layers:
            return "int4"
        p = _PROJ.search(name)
        if p is None:
            return "int4"
        proj = p.group("proj")
        if proj in self.SQINT2_PROJS:
            return "sqint2"
        if proj in self.INT3_PROJS:
            return "int3"
        return "int4"

    def kind_for(self, name: str, default: str = "q4a") -> str:
        f = self.format_for(name)
        return default if f is None else FORMAT_KIND[f]

    def summary(self, names) -> dict[str, int]:
        out = {"sqint2": 0, "int3": 0, "int4": 0, "skip": 0}
        for n in names:
            f = self.format_for(n)
            out["skip" if f is None else f] += 1
        return out

    def __repr__(self) -> str:
        return f"MixedPrecisionRouter(n_layers={self.n_layers}, boundary={sorted(self.boundary_layers)})"
