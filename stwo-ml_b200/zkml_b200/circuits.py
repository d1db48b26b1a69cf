"""Layer lists for zkml_prove_gkr_chain that mirror the engine's graph builders.

``hf_transformer_layers`` follows build_hf_transformer_graph (compiler/hf_loader.rs:770-813)
for a dense model with RMSNorm: per block RMSNorm, Q projection (d -> num_heads * head_dim),
O projection (-> d), RMSNorm, and the gated FFN as the linear chain the GKR walk proves
(GraphBuilder::gated_ffn, compiler/graph.rs:835-865: gate_proj d -> d_ff, the activation,
down_proj d_ff -> d); then a final RMSNorm.  As in the reference graph there are no K / V
projections, attention, RoPE, embedding or lm_head.  up_proj is not part of the circuit: the
reference multiplies it in only in forward passes given a named ``up_proj`` weight, and its
random-weight generator (compiler/onnx.rs:465-487) creates none.
"""
from typing import Callable, List, Tuple

import numpy as np


def hf_transformer_layers(d: int, q_dim: int, d_ff: int, n_blocks: int,
                          weight: Callable[[int, int, int], np.ndarray], activation: str = "silu") -> List[Tuple]:
    """The chain layers of ``n_blocks`` transformer blocks.  weight(index, rows, cols) returns
    the index-th weight matrix (rows x cols M31, row major) in graph order."""
    layers: List[Tuple] = []
    idx = 0

    def lin(rows, cols):
        nonlocal idx
        w = weight(idx, rows, cols)
        idx += 1
        return ("linear", w)

    for _ in range(n_blocks):
        layers.append(("rmsnorm", None))
        layers.append(lin(d, q_dim))
        layers.append(lin(q_dim, d))
        layers.append(("rmsnorm", None))
        layers.append(lin(d, d_ff))
        layers.append(("activation", activation))
        layers.append(lin(d_ff, d))
    layers.append(("rmsnorm", None))
    return layers
