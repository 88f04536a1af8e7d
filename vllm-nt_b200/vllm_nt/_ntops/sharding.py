"""How the hot path is partitioned across GPUs (one process per GPU).

* Paged decode shards by KV head: rank r of G owns KV heads [r*Hkv/G, (r+1)*Hkv/G) of the
  cache and the GQA group of query heads that read them.  Every rank processes all
  sequences; no data crosses GPUs inside attention, and the per-rank outputs are the
  head-slices of the full output.
* Projections follow vLLM's tensor parallelism: column-parallel (qkv, gate_up) split the
  weight rows (N); row-parallel (o_proj, down) split K and need a sum of the partial
  outputs across ranks (an all-reduce).
"""

from __future__ import annotations


def kv_head_range(rank: int, world: int, num_kv_heads: int) -> tuple[int, int]:
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads do not split evenly over {world} ranks")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def q_head_range(rank: int, world: int, num_q_heads: int, num_kv_heads: int) -> tuple[int, int]:
    """Query heads that read the KV heads of ``kv_head_range`` (GQA groups stay whole)."""
    group = num_q_heads // num_kv_heads
    h0, h1 = kv_head_range(rank, world, num_kv_heads)
    return h0 * group, h1 * group


def column_range(rank: int, world: int, n: int) -> tuple[int, int]:
    """Output features owned by a rank in a column-parallel projection."""
    if n % world:
        raise ValueError(f"N={n} does not split evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def row_range(rank: int, world: int, k: int) -> tuple[int, int]:
    """Input features owned by a rank in a row-parallel projection (partial sums are
    all-reduced)."""
    if k % world:
        raise ValueError(f"K={k} does not split evenly over {world} ranks")
    per = k // world
    return rank * per, (rank + 1) * per
