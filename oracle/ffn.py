"""CPU restatement of the reference FFN math (test infrastructure only).

The torch formulations repeat the reference's own ATen sequence so that, on
CPU, they reproduce its rounding: a bf16 input gives bf16 gate/up/activation
like runtime/ffn.py:26-31.  ``sparse_ffn_f64`` is the same math in numpy
float64 on the dtype-rounded weights, used as the tolerance anchor.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


def gather_weights(gate, up, down, ids):
    """runtime/ffn.py:20-23: selected gate rows, up rows and down columns."""
    if ids.ndim != 1:
        raise ValueError("batch-1 sparse runtime requires one-dimensional selected_ids")
    ids = ids.long()
    return gate.index_select(0, ids), up.index_select(0, ids), down.index_select(1, ids)


def packed_components(x, gate_sel, up_sel):
    """runtime/ffn.py:28-29: (gate, up, silu(gate) * up) in x's dtype."""
    g = F.linear(x, gate_sel)
    u = F.linear(x, up_sel)
    return g, u, F.silu(g) * u


def dynamic_sparse_ffn(x, ids, gate, up, down):
    """runtime/ffn.py:34-39 (TorchDynamicSparseFFN.forward)."""
    gs, us, ds = gather_weights(gate, up, down, ids)
    return F.linear(packed_components(x, gs, us)[2], ds)


def dynamic_sparse_activation(x, ids, gate, up):
    """Activation of the selected neurons, [B, K] (runtime/ffn.py:38)."""
    ids = ids.long()
    return packed_components(x, gate.index_select(0, ids), up.index_select(0, ids))[2]


def masked_dense(x, ids, gate, up, down):
    """runtime/ffn.py:42-43: dense gate/up, activation masked to ids, dense down."""
    g = F.linear(x, gate)
    u = F.linear(x, up)
    a = F.silu(g) * u
    mask = torch.zeros_like(a).scatter_(-1, ids.long().expand(x.shape[0], -1), 1)
    return F.linear(a * mask, down)


def sparse_ffn_f64(x, ids, gate, up, down, token_mask=None):
    """float64 numpy y[b] = sum_j m[j,b] silu(G_j.x_b)(U_j.x_b) D[:,j] on the given values."""
    xs = np.asarray(x.double().cpu().numpy())
    ids_np = np.asarray(ids.long().cpu().numpy())
    g = np.asarray(gate.double().cpu().numpy())[ids_np]
    u = np.asarray(up.double().cpu().numpy())[ids_np]
    d = np.asarray(down.double().cpu().numpy())[:, ids_np]
    gv = xs @ g.T
    uv = xs @ u.T
    a = gv / (1.0 + np.exp(-gv)) * uv
    if token_mask is not None:
        bits = np.asarray(token_mask.cpu().numpy()).astype(np.int64)
        use = (bits[None, :] >> np.arange(xs.shape[0])[:, None]) & 1
        a = a * use
    return a @ d.T


def reconstruct(activations, down, indices, bias=None):
    """oracle/sparse_ffn.py:8-13: per-row W[:, S] a[S] via scatter into zeros."""
    selected = torch.zeros_like(activations)
    selected.scatter_(1, indices.long(), activations.gather(1, indices.long()))
    return F.linear(selected, down, bias)


def importance_scores(activations, down, metric):
    """oracle/importance.py:6-18."""
    if activations.shape[-1] != down.shape[1]:
        raise ValueError("activation width must equal down-projection input width")
    if metric in {"activation", "activation_magnitude"}:
        return activations.abs()
    norms = torch.linalg.vector_norm(down.float(), dim=0)
    if metric in {"weighted_activation", "weighted_contribution"}:
        return activations.abs().float() * norms
    if metric in {"exact", "exact_output_norm"}:
        return (activations.float().square() * down.float().square().sum(dim=0)).sqrt()
    raise ValueError(f"Unknown importance metric {metric!r}")


def pack_records(gate: np.ndarray, up: np.ndarray, down: np.ndarray) -> np.ndarray:
    """Neuron-major records [gate[n,:Hp] | up[n,:Hp] | down[:Hp,n]] (zero padded to Hp = ceil8(H))."""
    n, h = gate.shape
    hp = (h + 7) // 8 * 8
    out = np.zeros((n, 3 * hp), dtype=gate.dtype)
    out[:, :h] = gate
    out[:, hp:hp + h] = up
    out[:, 2 * hp:2 * hp + h] = down.T
    return out


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den > 0 else float(np.linalg.norm(a - b))
