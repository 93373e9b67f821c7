"""The token-cached prefix scan (ews/core/token_scan.py:55-118) on the B200 engines.

With a finite vocabulary, segment t of a token sequence has the displacement vocab_dx[g_t] (already lifted)
and the clock increment vocab_dtheta[g_t] of its token g_t. The reference caches every token's local
signature and flow and runs a sequential scan gathering them by token. The engines evaluate the local terms
and the flows in-kernel from per-interval increments and clock steps, so here the cache is the vocabulary
itself: the sequence's increments and clock knots are gathered (a padded step gets a zero displacement and a
zero clock step, i.e. the identity flow and the unit signature, as the reference's mask does) and the layer's
per-interval-clock engine (diagonal or 2x2-block A) runs the prefix scan, forward and backward.
"""

from __future__ import annotations

from typing import Optional

import torch


def token_cached_prefix(layer, token_ids: torch.Tensor, vocab_dx: torch.Tensor, vocab_dtheta: torch.Tensor,
                        mask: Optional[torch.Tensor] = None, a_scale=1.0) -> torch.Tensor:
    """Prefix levels of token sequences, the reference's ``token_cached_prefix_scan(build_token_cache(...))``.

    layer: an ``EWS`` with ``reweighting_mode="displacement"`` (the per-token clock steps are its intervals'
    steps); token_ids (L,) or (B, L) integers; vocab_dx (V, d) lifted displacements (d = the layer's state
    dimension); vocab_dtheta (V,); mask (L,) / (B, L) bool or None. Returns (L, D) / (B, L, D), D = sum_k d^k,
    the packed levels after each token (level 0 dropped), differentiable in vocab_dx, vocab_dtheta and A."""
    if layer.reweighting_mode != "displacement":
        raise ValueError("the token-cached scan takes one clock step per token: use reweighting_mode='displacement'")
    single = token_ids.dim() == 1
    tok = token_ids[None] if single else token_ids
    dx = vocab_dx[tok]  # (B, L, d)
    dth = vocab_dtheta[tok]  # (B, L)
    if mask is not None:
        m = (mask[None] if single else mask).to(dx.dtype)
        dx = dx * m[..., None]
        dth = dth * m
    clock = torch.cat([torch.zeros_like(dth[:, :1]), torch.cumsum(dth, -1)], -1)
    out = layer(dx, clock, readout="prefix", increments=True, a_scale=a_scale)[..., 1:]
    return out[0] if single else out
