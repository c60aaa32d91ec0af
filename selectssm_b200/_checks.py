"""Argument rules of the reference's scan selectors, free of any array library,
so the PyTorch host (ops.py) and the JAX binding (jax_ffi.py) share them and the
JAX binding loads without PyTorch."""

from __future__ import annotations

import math


def largest_factor_up_to(b, n):
    """selectssm.py:24-30: largest k <= b dividing n (n itself when n < 2)."""
    if n < 2:
        return n
    k = b
    while n % k != 0:
        k -= 1
    return k


def check_chunked(L, D, chunk_size, n_channel_groups):
    """The ValueErrors of selectssm.py:47-48 and :53-54; returns the chunk size
    the reference would use (selectssm.py:50-51)."""
    K = 1 if n_channel_groups is None else n_channel_groups
    if D % K != 0:
        raise ValueError(f"n_channel_groups={n_channel_groups} must divide D={D}")
    if chunk_size is None:
        chunk_size = largest_factor_up_to(int(math.sqrt(K * L)), L)
    if L % chunk_size != 0:
        raise ValueError(f"chunk_size={chunk_size} must divide L={L}")
    return chunk_size
