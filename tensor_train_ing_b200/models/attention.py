"""Dense attention math: the authoritative (oracle) definitions the fused kernels are tested against.

Polynomial attention (reference tnlm/attention.py:48-77) for queries i and keys j:

    S_ij = q_i . k_j / sqrt(d_k)
    signed_product    A = S1 * S2
    offset_square     A = (S1 + b_h)^2
    lower_degree_mix  A = c0 + c1 S1 + c2 S2 + c12 S1 S2
    y_i = sum_j C_ij A_ij v_j,   C = visible * n_visible^-p

"visible" = causal, same document, query and key both real tokens (doc id >= 0).  The mask is
applied after the polynomial (a zero, never -inf) and there is no softmax.  The softmax control
and the exact recurrent form of ``signed_product`` are kept as well.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def doc_positions(doc_ids: torch.Tensor) -> torch.Tensor:
    """Position of every token inside its (contiguous) document, shape (B, T)."""
    B, T = doc_ids.shape
    t = torch.arange(T, device=doc_ids.device).expand(B, T)
    new_doc = torch.ones_like(doc_ids, dtype=torch.bool)
    new_doc[:, 1:] = doc_ids[:, 1:] != doc_ids[:, :-1]
    start = torch.where(new_doc, t, torch.zeros_like(t)).cummax(dim=-1).values
    return t - start


def visible_mask(doc_ids: torch.Tensor) -> torch.Tensor:
    """(B, 1, T, T) bool: key j is visible from query i.  Padding (doc id < 0) sees nothing and is
    seen by nothing, so padding rows come out exactly zero."""
    T = doc_ids.shape[1]
    causal = torch.ones(T, T, dtype=torch.bool, device=doc_ids.device).tril()
    real = doc_ids >= 0
    same_doc = doc_ids.unsqueeze(2) == doc_ids.unsqueeze(1)
    return (causal & same_doc & real.unsqueeze(2) & real.unsqueeze(1)).unsqueeze(1)


def row_scale_mask(visible: torch.Tensor, power: float, dtype=torch.float32) -> torch.Tensor:
    """C = visible * n_visible^-power (empty rows stay zero)."""
    n = visible.sum(dim=-1, keepdim=True).clamp_min(1).to(dtype)
    return visible.to(dtype) * n.pow(-power)


def row_scale_vector(doc_ids: torch.Tensor, power: float) -> torch.Tensor:
    """The same scale as a (B, T) vector for contiguous documents: (pos + 1)^-p, 0 for padding."""
    n = (doc_positions(doc_ids) + 1).float()
    return torch.where(doc_ids >= 0, n.pow(-power), torch.zeros_like(n))


def rope_inv_freq(dim: int, base: float, device=None) -> torch.Tensor:
    """Rotation frequencies 1 / base^(2i/dim), i < dim/2 (fp32, the rounding the reference uses)."""
    return 1.0 / (base ** (torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim))


def rope_tables(positions: torch.Tensor, dim: int, base: float):
    """cos/sin tables of shape (B, 1, T, dim/2) for the half-split rotary embedding."""
    angle = positions.float().unsqueeze(-1) * rope_inv_freq(dim, base, positions.device)
    return angle.cos().unsqueeze(1), angle.sin().unsqueeze(1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate feature pairs (i, i + d/2) by the position angle; computed in >= fp32."""
    xf = x.to(torch.promote_types(x.dtype, torch.float32))
    half = xf.shape[-1] // 2
    a, b = xf[..., :half], xf[..., half:]
    return torch.cat((a * cos - b * sin, a * sin + b * cos), dim=-1).to(x.dtype)


def scores(q: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    return torch.matmul(q, k.transpose(-1, -2)) * (q.shape[-1] ** -0.5)


def polynomial_scores(kind: str, S1, S2=None, coef=None, b=None):
    if kind == "signed_product":
        return S1 * S2
    if kind == "offset_square":
        return (S1 + b.view(1, -1, 1, 1)) ** 2
    if kind == "lower_degree_mix":
        c0, c1, c2, c12 = (coef[:, i].view(1, -1, 1, 1) for i in range(4))
        return c0 + c1 * S1 + c2 * S2 + c12 * S1 * S2
    raise ValueError(f"unknown polynomial attention kind {kind!r}")


def polynomial_attention(kind: str, q1, k1, q2, k2, v, C, coef=None, b=None):
    """Dense oracle.  q*, k*: (B, H, T, dk); v: (B, H, T, dv); C: (B, 1|H, T, T)."""
    S1 = scores(q1, k1)
    S2 = scores(q2, k2) if kind in ("signed_product", "lower_degree_mix") else None
    P = C * polynomial_scores(kind, S1, S2, coef, b)
    return torch.matmul(P.to(v.dtype), v)


def polynomial_attention_recurrent(q1, k1, q2, k2, v, scale):
    """Exact O(T dk^2 dv) recurrent form of ``signed_product`` for one document.

    state_t = state_{t-1} + (k1_t (x) k2_t) v_t^T,   y_t = scale_t (q1_t (x) q2_t)^T state_t / dk
    Shapes (H, T, d); ``scale`` is the (T,) row scale.  Used as an oracle only.
    """
    H, T, dk = q1.shape
    state = q1.new_zeros(H, dk * dk, v.shape[-1])
    out = []
    for t in range(T):
        kk = torch.einsum("hi,hj->hij", k1[:, t], k2[:, t]).reshape(H, -1)
        state = state + kk.unsqueeze(-1) * v[:, t].unsqueeze(1)
        qq = torch.einsum("hi,hj->hij", q1[:, t], q2[:, t]).reshape(H, -1)
        out.append(torch.einsum("hs,hsv->hv", qq, state) * (scale[t] / dk))
    return torch.stack(out, dim=1)


def softmax_attention(q, k, v, visible):
    """Softmax control on a dense mask; rows with nothing visible output exactly zero."""
    has_key = visible.any(dim=-1, keepdim=True)
    T = visible.shape[-1]
    diag = torch.eye(T, dtype=torch.bool, device=visible.device)
    y = F.scaled_dot_product_attention(q, k, v, attn_mask=visible | (~has_key & diag))
    return y * has_key.to(y.dtype)


_FLEX_COMPILED = None


def softmax_attention_flex(q, k, v, doc_ids):
    """Softmax control through FlexAttention with a causal + same-document block mask.

    The softmax control model is a comparison baseline, not a tensor-network hot path, so it
    uses PyTorch's FlexAttention (compiled once) rather than a hand-written kernel."""
    global _FLEX_COMPILED
    from torch.nn.attention.flex_attention import create_block_mask, flex_attention
    B, T = doc_ids.shape
    docs = doc_ids

    def mask_mod(b, h, qi, ki):
        return (qi >= ki) & (docs[b, qi] == docs[b, ki]) & (docs[b, ki] >= 0)

    block_mask = create_block_mask(mask_mod, B, None, T, T, device=q.device)
    if _FLEX_COMPILED is None:
        _FLEX_COMPILED = torch.compile(flex_attention, dynamic=False)
    y = _FLEX_COMPILED(q, k, v, block_mask=block_mask)
    return y * (doc_ids >= 0)[:, None, :, None].to(y.dtype)
