"""Reverse-complement parameter sharing (RCPS) around the scan modules.

Mirror of src/selectssm/rcps.py for PyTorch.  The group action is
RC(x)[b, l, d] = x[b, L-1-l, D-1-d] (rcps.py:37-39).  A (B, L, 2D) tensor
carries the sense strand in channels [0, D) and the antisense strand in
[D, 2D); shared weights process both.

Difference from the reference, with the same result: RCPSWrapper
(rcps.py:42-72) calls its inner module twice, once per strand, on a flipped
copy of the antisense strand.  Here a forward SelectiveSSM inner module runs
the antisense strand through its reversed, complemented in-place read
(SelectiveSSM.forward_rc), so no flipped copy is made; any other inner module
gets the sense strand and the conjugated antisense strand stacked along the
batch axis and runs once on 2B rows.  This relies on the inner module treating batch rows
independently, which SelectiveSSM, BidirectionalMamba and every norm here do.
"""

from __future__ import annotations

from typing import Sequence

import torch
import torch.nn as nn

from .modules import _RMSNorm, _lecun_normal_


def rc_conjugate(x: torch.Tensor) -> torch.Tensor:
    """Flip the sequence and channel axes (rcps.py:37-39)."""
    return torch.flip(x, dims=(-2, -1))


class RCPSWrapper(nn.Module):
    """RC-equivariant wrapper of a (B, L, D) -> (B, L, D) module (rcps.py:42-72).

    Input and output are (B, L, 2D).  ``module`` is the inner module (shared
    by both strands); the reference builds it from ``module_cls(**module_kwargs)``,
    which ``from_cls`` reproduces.
    """

    def __init__(self, module: nn.Module):
        super().__init__()
        self.inner = module

    @classmethod
    def from_cls(cls, module_cls, module_kwargs: dict | None = None):
        return cls(module_cls(**(module_kwargs or {})))

    def forward(self, x: torch.Tensor, **kwargs) -> torch.Tensor:
        D = x.shape[-1] // 2
        sense, antisense = x[..., :D], x[..., D:]
        rc_inner = getattr(self.inner, "forward_rc", None)
        if rc_inner is not None and not (self.inner.reverse or self.inner.complement):
            # a forward SelectiveSSM reads the antisense strand reversed and
            # complemented in place (no flipped copies in or out)
            return torch.cat([self.inner(sense, **kwargs), rc_inner(antisense, **kwargs)], dim=-1)
        both = torch.cat([sense, rc_conjugate(antisense)], dim=0)  # (2B, L, D): one inner call
        out = self.inner(both, **kwargs)
        B = x.shape[0]
        return torch.cat([out[:B], rc_conjugate(out[B:])], dim=-1)


class RCPSNorm(nn.Module):
    """RC-equivariant normalisation with one shared norm (rcps.py:75-100);
    ``norm`` defaults to RMSNorm (flax.linen.RMSNorm) of width D."""

    def __init__(self, d: int, norm: nn.Module | None = None):
        super().__init__()
        self.norm = norm if norm is not None else _RMSNorm(d)

    def forward(self, x: torch.Tensor, **kwargs) -> torch.Tensor:
        D = x.shape[-1] // 2
        sense = self.norm(x[..., :D], **kwargs)
        antisense = rc_conjugate(self.norm(rc_conjugate(x[..., D:]), **kwargs))
        return torch.cat([sense, antisense], dim=-1)


class RCPSEmbedding(nn.Module):
    """Token ids (B, L) -> (B, L, 2 d_model): the sense embedding and the
    conjugated embedding of the reverse-complemented ids (rcps.py:103-136)."""

    def __init__(self, vocab_size: int, d_model: int, complement_map: Sequence[int]):
        super().__init__()
        self.embed = nn.Embedding(vocab_size, d_model)
        # flax nn.Embed's default init: variance scaling 1 / features, normal
        nn.init.normal_(self.embed.weight, std=d_model ** -0.5)
        self.register_buffer("cmap", torch.as_tensor(list(complement_map), dtype=torch.long), persistent=False)

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        sense = self.embed(input_ids)
        rc_ids = torch.flip(self.cmap[input_ids], dims=(-1,))
        antisense = rc_conjugate(self.embed(rc_ids))
        return torch.cat([sense, antisense], dim=-1)


class RCPSLMHead(nn.Module):
    """(B, L, 2D) -> (B, L, vocab) logits summing the sense projection and the
    channel-flipped antisense projection with complement-reindexed weights
    (rcps.py:139-172).  Parameters ``kernel`` (D, vocab) and ``bias`` (vocab)
    use the reference's names and layout."""

    def __init__(self, d: int, vocab_size: int, complement_map: Sequence[int]):
        super().__init__()
        self.kernel = nn.Parameter(_lecun_normal_(torch.empty(d, vocab_size), d))
        self.bias = nn.Parameter(torch.zeros(vocab_size))
        self.register_buffer("cmap", torch.as_tensor(list(complement_map), dtype=torch.long), persistent=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        D = x.shape[-1] // 2
        sense, antisense = x[..., :D], x[..., D:]
        fwd_logits = sense @ self.kernel + self.bias
        rc_logits = torch.flip(antisense, dims=(-1,)) @ self.kernel[:, self.cmap] + self.bias
        return fwd_logits + rc_logits
