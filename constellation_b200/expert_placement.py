"""Expert-id helpers with the interface of the reference's ``server/expert_placement.py``.

Global expert id = ``layer * experts_per_layer + local`` (``make_global_expert_id``,
``server/expert_placement.py:4-25``) and its inverse (``:28-40``); the resident local
ids of one layer (``:43-59``); lookup of a placement record (``:62-67``) and grouping
by control endpoint (``:70-79``).  Same names, arguments, results and ``ValueError`` /
``RuntimeError`` behaviour, so callers switch modules without change.  Added: the
expert-parallel owner rule used by ``constellation_b200.ep``.
"""
from __future__ import annotations

from typing import Iterable


def make_global_expert_id(layer_id: int, local_expert_id: int, experts_per_layer: int = 256) -> int:
    layer_id, local_expert_id, experts_per_layer = int(layer_id), int(local_expert_id), int(experts_per_layer)
    if layer_id < 0:
        raise ValueError(f"layer_id must be >= 0, got {layer_id}")
    if local_expert_id < 0:
        raise ValueError(f"local_expert_id must be >= 0, got {local_expert_id}")
    if experts_per_layer <= 0:
        raise ValueError(f"experts_per_layer must be > 0, got {experts_per_layer}")
    if local_expert_id >= experts_per_layer:
        raise ValueError(f"local_expert_id must be < experts_per_layer, got "
                         f"{local_expert_id} vs {experts_per_layer}")
    return layer_id * experts_per_layer + local_expert_id


def split_global_expert_id(global_expert_id: int, experts_per_layer: int = 256) -> tuple[int, int]:
    global_expert_id, experts_per_layer = int(global_expert_id), int(experts_per_layer)
    if global_expert_id < 0:
        raise ValueError(f"global_expert_id must be >= 0, got {global_expert_id}")
    if experts_per_layer <= 0:
        raise ValueError(f"experts_per_layer must be > 0, got {experts_per_layer}")
    return divmod(global_expert_id, experts_per_layer)


def allowed_local_expert_ids_for_layer(global_expert_ids: Iterable[int], layer_id: int,
                                       experts_per_layer: int = 256) -> list[int]:
    layer_id = int(layer_id)
    found = set()
    for gid in global_expert_ids:
        lay, loc = split_global_expert_id(int(gid), experts_per_layer=experts_per_layer)
        if lay == layer_id:
            found.add(loc)
    return sorted(found)


def find_expert_placement(placements, expert_id: int):
    expert_id = int(expert_id)
    for p in placements:
        if int(p["expert_id"]) == expert_id:
            return p
    raise RuntimeError(f"expert {expert_id} not found in placements")


def group_placements_by_control_endpoint(placements):
    groups: dict = {}
    for p in placements:
        groups.setdefault((str(p["host"]), int(p["control_port"])), []).append(p)
    for v in groups.values():
        v.sort(key=lambda p: int(p["expert_id"]))
    return groups


def ep_owner_rank(local_expert_id: int, n_routed_experts: int, world: int) -> int:
    """Rank that holds ``local_expert_id`` when ``n_routed_experts`` are split into
    ``world`` contiguous blocks (``rank_begin = ep_rank * experts_per_rank``)."""
    if n_routed_experts % world:
        raise ValueError(f"{n_routed_experts} experts do not shard over {world} ranks")
    return int(local_expert_id) // (n_routed_experts // world)
