"""Expert-parallel partition and exchange layout (host side).

Experts are sharded by id: expert e of every layer lives on rank
``e % world``.  Per layer and token every rank knows the route (ids, w) --
the router runs redundantly on every rank from the same logits -- computes
the down outputs y_s of the slots it owns into ``contrib[slot][hidden]``,
and one all-gather builds ``gathered[rank][slot][hidden]``.  The route-order
sum then reads slot s from rank ``owner(ids[s])``, so every rank ends with
the same x_{L+1}, bit-identical to one GPU (the reference is single-GPU;
its route-order contract is runtime.py:588-596).
"""

from __future__ import annotations


def owner(expert: int, world: int) -> int:
    return int(expert) % int(world)


def owned_slots(ids, world: int, rank: int) -> list[int]:
    return [s for s, e in enumerate(ids) if owner(int(e), world) == rank]


def gathered_index(ids, slot: int, world: int, top_k: int, hidden: int) -> int:
    """Flat offset of slot `slot`'s output in the gathered buffer."""
    return (owner(int(ids[slot]), world) * top_k + slot) * hidden


def experts_of_rank(n_experts: int, world: int, rank: int) -> list[int]:
    return list(range(rank, n_experts, world))
