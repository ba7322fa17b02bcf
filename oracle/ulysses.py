"""Ulysses all-to-all oracle (TEST INFRASTRUCTURE, see oracle/__init__.py).

Restates wan_5b/distributed/util.py:52-64 `all_to_all(x, scatter_dim,
gather_dim)` for all ranks at once: rank r splits its x into P chunks along
scatter_dim, chunk j goes to rank j, and rank j concatenates what it receives
(in source-rank order) along gather_dim.  Used as in ulysses.py:40-54:
seq -> head (scatter heads, gather sequence) before attention, head -> seq after.
"""
import numpy as np


def all_to_all(xs, scatter_dim, gather_dim):
    P = len(xs)
    parts = [np.split(x, P, axis=scatter_dim) for x in xs]
    return [np.concatenate([parts[src][dst] for src in range(P)], axis=gather_dim) for dst in range(P)]


def seq_to_head(xs):
    """[B, L/P, H, D] per rank -> [B, L, H/P, D] per rank."""
    return all_to_all(xs, scatter_dim=2, gather_dim=1)


def head_to_seq(xs):
    """[B, L, H/P, D] per rank -> [B, L/P, H, D] per rank."""
    return all_to_all(xs, scatter_dim=1, gather_dim=2)
