"""Long contexts without a T x T score matrix: polynomial attention in linear-state (chunked
recurrent) form, and its exact context-parallel split over ranks.

The reference has only a per-token recurrent oracle (tnlm/attention.py:80-95).  Polynomial
attention has no softmax, so every kind factors through feature maps of queries and keys:

    A(S1, S2) = phi_q(q) . phi_k(k),   S = q . k / sqrt(d_k)

    signed_product    phi_q = s q1 (x) s q2               phi_k = k1 (x) k2
    offset_square     phi_q = [s q (x) s q, 2 b s q, b^2]  phi_k = [k (x) k, k, 1]
    lower_degree_mix  phi_q = [c0, c1 s q1, c2 s q2, c12 s q1 (x) s q2]
                      phi_k = [1, k1, k2, k1 (x) k2]          (s = d_k^-1/2; b, c per head)

so y_i = scale_i * phi_q(q_i) . sum_{j visible} phi_k(k_j) v_j^T.  With contiguous documents the
visible keys of a query are the earlier tokens of its own document, so a running state
sum phi_k(k) v^T, reset where a document starts, gives the exact output.  ``chunked_polynomial_attention``
takes the sequence in chunks: inside a chunk the causal same-document part is a small dense
product, and queries of the document that was open at the chunk's start add phi_q . state.  The
state has F x d_v entries per head (F = d_k^2 for the products), so the form pays off when T is well
beyond F / d_k, or when the sequence is split over GPUs:

``context_parallel_attention`` gives each rank a contiguous slice of every row.  A rank's slice
summarises to the state of its last document segment plus whether the slice lies inside a single
document; the ranks exchange these summaries (one all-gather of F x d_v per head and row, independent
of T), each folds the summaries of the ranks before it into the state entering its slice, and runs
the chunked form from there.  The result equals the dense attention over the whole row, and the
all-gather is differentiable, so it trains.
"""
from __future__ import annotations

import torch


def _outer(a, b):
    return (a.unsqueeze(-1) * b.unsqueeze(-2)).flatten(-2)


def query_features(kind: str, q1, q2=None, coef=None, b=None):
    """phi_q of shape (B, H, T, F)."""
    s = q1.shape[-1] ** -0.5
    ones = torch.ones_like(q1[..., :1])
    if kind == "signed_product":
        return _outer(q1 * s, q2 * s)
    if kind == "offset_square":
        bh = b.view(1, -1, 1, 1).to(q1.dtype)
        return torch.cat([_outer(q1 * s, q1 * s), 2 * bh * q1 * s, (bh * bh) * ones], dim=-1)
    if kind == "lower_degree_mix":
        c0, c1, c2, c12 = (coef[:, i].view(1, -1, 1, 1).to(q1.dtype) for i in range(4))
        return torch.cat([c0 * ones, c1 * q1 * s, c2 * q2 * s, c12 * _outer(q1 * s, q2 * s)], dim=-1)
    raise ValueError(f"no linear-state form for attention kind {kind!r}")


def key_features(kind: str, k1, k2=None):
    """phi_k of shape (B, H, T, F)."""
    ones = torch.ones_like(k1[..., :1])
    if kind == "signed_product":
        return _outer(k1, k2)
    if kind == "offset_square":
        return torch.cat([_outer(k1, k1), k1, ones], dim=-1)
    if kind == "lower_degree_mix":
        return torch.cat([ones, k1, k2, _outer(k1, k2)], dim=-1)
    raise ValueError(f"no linear-state form for attention kind {kind!r}")


def feature_maps(kind: str, q1, k1, q2=None, k2=None, coef=None, b=None):
    """(phi_q, phi_k) with A(S1, S2) = phi_q . phi_k for each head."""
    return query_features(kind, q1, q2, coef, b), key_features(kind, k1, k2)


def _segment_state(phi_k, v, keep):
    """sum over the kept keys of phi_k v^T: (B, H, F, dv)."""
    return (phi_k * keep.unsqueeze(1).unsqueeze(-1).to(phi_k.dtype)).transpose(-1, -2) @ v


def chunked_polynomial_attention(kind, q1, k1, q2, k2, v, doc_ids, scale, *, chunk: int = 256, coef=None, b=None,
                                 state=None, state_doc=None):
    """Exact polynomial attention in chunks of ``chunk`` tokens.

    q*, k*: (B, H, T, dk); v: (B, H, T, dv); doc_ids: (B, T) contiguous documents (negative =
    padding, which sees and is seen by nothing); scale: (B, T) row scale.  ``state`` /
    ``state_doc``: the running state (B, H, F, dv) of the document ``state_doc`` (B,) open before
    the first token (context parallelism); zeros / no document when omitted.
    Returns (y (B, H, T, dv), final state, final state's document)."""
    phi_q, phi_k = feature_maps(kind, q1, k1, q2, k2, coef, b)
    B, H, T, F = phi_q.shape
    if state is None:
        state = phi_q.new_zeros(B, H, F, v.shape[-1])
        state_doc = torch.full((B,), -1, dtype=doc_ids.dtype, device=doc_ids.device)
    out = []
    for c0 in range(0, T, chunk):
        sl = slice(c0, min(T, c0 + chunk))
        d = doc_ids[:, sl]
        real = d >= 0
        causal = torch.ones(d.shape[1], d.shape[1], dtype=torch.bool, device=d.device).tril()
        visible = causal & (d.unsqueeze(2) == d.unsqueeze(1)) & real.unsqueeze(2) & real.unsqueeze(1)
        pq, pk, vc = phi_q[:, :, sl], phi_k[:, :, sl], v[:, :, sl]
        inner = (pq @ pk.transpose(-1, -2)) * visible.unsqueeze(1).to(pq.dtype)
        carried = (d == state_doc.unsqueeze(1)) & real
        y = inner @ vc + (pq @ state) * carried.unsqueeze(1).unsqueeze(-1).to(pq.dtype)
        out.append(y * scale[:, sl].unsqueeze(1).unsqueeze(-1).to(y.dtype))
        last = d[:, -1]
        tail = _segment_state(pk, vc, (d == last.unsqueeze(1)) & real)
        continues = (last == state_doc) & (last >= 0)
        state = torch.where(continues.view(B, 1, 1, 1), state + tail, tail)
        state_doc = last
    return torch.cat(out, dim=2), state, state_doc


def slice_summary(kind, k1, k2, v, doc_ids):
    """What a slice contributes to later slices: the state of its last document segment, that
    document, and whether the whole slice belongs to it (so earlier state flows through)."""
    phi_k = key_features(kind, k1, k2)
    last = doc_ids[:, -1]
    keep = (doc_ids == last.unsqueeze(1)) & (doc_ids >= 0)
    whole = keep.all(dim=1)
    return _segment_state(phi_k, v, keep), last, whole


def fold_summaries(states, docs, wholes, upto: int):
    """The state entering slice ``upto`` from the summaries of slices 0 .. upto-1 (in order)."""
    state = torch.zeros_like(states[0])
    doc = torch.full_like(docs[0], -1)
    for r in range(upto):
        continues = wholes[r] & (docs[r] == doc) & (docs[r] >= 0)
        state = torch.where(continues.view(-1, 1, 1, 1), state + states[r], states[r])
        doc = docs[r]
    return state, doc


def context_parallel_attention(kind, q1, k1, q2, k2, v, doc_ids, scale, *, group=None, chunk: int = 256,
                               coef=None, b=None):
    """Exact polynomial attention over rows split into contiguous slices, one per rank of
    ``group`` in rank order.  Each argument holds this rank's slice; ``doc_ids`` and ``scale`` must
    be the global values for it (a document crossing a slice boundary keeps one id, and the row
    scale uses the position inside the whole document)."""
    import torch.distributed as dist
    from torch.distributed.nn.functional import all_gather
    rank = dist.get_rank(group)
    state, last, whole = slice_summary(kind, k1, k2, v, doc_ids)
    states = all_gather(state.contiguous(), group=group)
    docs = [torch.empty_like(last) for _ in states]
    wholes = [torch.empty_like(whole) for _ in states]
    dist.all_gather(docs, last.contiguous(), group=group)
    dist.all_gather(wholes, whole.contiguous(), group=group)
    entering, entering_doc = fold_summaries(states, docs, wholes, rank)
    # every rank's graph must reach the gathered states, or the ranks that use none of them (rank 0)
    # would skip the gather's backward collective that the others enter
    entering = entering + 0.0 * torch.stack(list(states)).sum(dim=0)
    y, _, _ = chunked_polynomial_attention(kind, q1, k1, q2, k2, v, doc_ids, scale, chunk=chunk, coef=coef, b=b,
                                           state=entering, state_doc=entering_doc)
    return y
