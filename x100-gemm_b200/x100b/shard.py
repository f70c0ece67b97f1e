"""How the hot path is split over the GPUs of one node (one process each).

* GEMM: B and C are split by columns (N-sharding); every rank holds all of A
  and computes C[:, n0:n1] = A . B[:, n0:n1] with no exchange.
* MoE layer: expert parallel.  Rank r holds experts [lo, hi) and the full
  router, so every rank selects the same top-k without an exchange; each rank
  returns the weighted sum over its local selected experts and the layer
  output is the sum over ranks (one all-reduce of batch x d floats).
"""
from __future__ import annotations


def gemm_cols(N: int, world: int, rank: int) -> tuple[int, int]:
    """Column range [n0, n1) of B and C owned by `rank` (N must divide by world)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if N % world:
        raise ValueError(f"N={N} does not divide over {world} ranks")
    w = N // world
    return rank * w, (rank + 1) * w


def expert_slice(n_exp: int, world: int, rank: int) -> tuple[int, int]:
    """Experts [lo, hi) held by `rank`; the slices cover [0, n_exp) exactly."""
    if world < 1 or not 0 <= rank < world or world > n_exp:
        raise ValueError(f"rank {rank} of world {world} for {n_exp} experts")
    return rank * n_exp // world, (rank + 1) * n_exp // world
