"""Work partition of one prefill op across GPUs (one process per GPU, no data-path collective).

Every stage of the op is independent per (batch, kv head) -- the q heads of a kv head share its
keys -- and, inside a head, per query tile: a tile's row maxima, votes, selection and attention
read only its own queries and the keys before them (shared_selection_triton_exact_2.py:69-92,
:291 and :169 take the absolute query position ``q_pos_base + row``).  So a layer splits into
units (kv-head range, query slab) whose results are exactly the whole-layer results, with no
exchange between ranks:

* ``heads``: each rank takes an equal range of kv heads (and their q heads) over the whole
  sequence;
* ``slabs``: each rank takes every head and one contiguous slab of query positions
  [start, end), called with k / v truncated to the first ``end`` keys and ``q_pos_base=start``;
  slab edges are multiples of 128 placed so the causal cost is balanced;
* ``grid``: heads split into ``gcd(kv_heads, world)`` parts, each part's sequence into
  ``world / parts`` slabs.

Keys are replicated rather than split: one sequence's K and V (bf16, 8 kv heads, 128k keys,
head_dim 128) is 0.5 GB, small beside a B200's 180 GB, and replicating them removes the
row-max all-reduce, the vote-count exchange and the partial-softmax merge a key split needs.
"""
from __future__ import annotations

import math

ALIGN = 128  # query slab edges: the tensor-core selection kernel's 128-row query block


def kv_head_range(n_kv_heads: int, parts: int, part: int):
    """[k0, k1) kv heads of part ``part`` out of ``parts`` equal parts."""
    if n_kv_heads % parts:
        raise ValueError(f"{n_kv_heads} kv heads do not split into {parts} equal parts")
    return part * n_kv_heads // parts, (part + 1) * n_kv_heads // parts


def slab_edges(n: int, parts: int, attend_weight: float = 4096.0, align: int = ALIGN):
    """Edges 0 = e_0 < ... < e_parts = n of query slabs with balanced cost.

    The cost of the query at position x is modelled as x + attend_weight: the selection
    kernel's two passes scale with the x causal keys, the attend stage with the kept set
    (bounded by k_max, roughly constant).  Slab r ends where the cumulative cost
    x^2 / 2 + attend_weight * x reaches r / parts of the total; edges are rounded to
    multiples of ``align`` and kept strictly increasing where n allows."""
    if parts < 1:
        raise ValueError("parts must be >= 1")
    total = n * n / 2.0 + attend_weight * n
    edges = [0]
    for r in range(1, parts):
        c = total * r / parts
        x = -attend_weight + math.sqrt(attend_weight * attend_weight + 2.0 * c)
        e = int(round(x / align)) * align
        e = max(e, edges[-1] + align)
        edges.append(min(e, n))
    edges.append(n)
    for a, b in zip(edges, edges[1:]):
        if b <= a:
            raise ValueError(f"sequence of {n} positions is too short for {parts} slabs")
    return edges


def plan(n_kv_heads: int, n: int, world: int, rank: int, mode: str = "heads",
         attend_weight: float = 4096.0):
    """Unit of rank ``rank``: dict(kv=(k0, k1), slab=(start, end), mode=...)."""
    if mode == "auto":
        mode = "heads" if n_kv_heads % world == 0 else "grid"
    if mode == "heads":
        hp, sp = world, 1
    elif mode == "slabs":
        hp, sp = 1, world
    elif mode == "grid":
        hp = math.gcd(n_kv_heads, world)
        sp = world // hp
    else:
        raise ValueError(mode)
    hpart, spart = rank // sp, rank % sp
    kv = kv_head_range(n_kv_heads, hp, hpart)
    edges = slab_edges(n, sp, attend_weight)
    return {"kv": kv, "slab": (edges[spart], edges[spart + 1]), "mode": mode,
            "head_parts": hp, "slab_parts": sp}
