"""Multi-GPU placement of a scene batch: scene sharding and camera splitting.

Scenes are independent (per-scene parameters, per-(scene, camera) images), so a batch
of S scenes shards by scene over the ranks of one node with no communication in the
render step: each rank renders a contiguous block of scenes.  When there are more
ranks than scenes, each scene is given a group of ranks; every rank of the group
renders a contiguous range of the scene's cameras against a full replica of the
scene's parameters, and after backward the group sums the parameter gradients with
one NCCL all-reduce over a single flattened fp32 bucket (over NVLink/NVSwitch; NVLS
reduces in the switch when NCCL enables it).  One process per GPU; torch.distributed
provides the process groups.

The reference renders every scene and camera of a call on one device and has no
multi-GPU code; this module is the B200 build's addition for batched workloads.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

# per-(scene, camera) inputs of the public renderers; everything else is per scene
PER_CAMERA = ("view_matrices", "intrinsics", "backgrounds")


def block(count: int, rank: int, world: int) -> slice:
    """Contiguous block partition of ``count`` items: rank r gets [r*count//world, ...)."""
    return slice(rank * count // world, (rank + 1) * count // world)


@dataclass(frozen=True)
class Shard:
    """What one rank renders: a scene range, a camera range, and its gradient group."""

    scenes: slice
    cameras: slice
    group_ranks: tuple[int, ...]     # ranks sharing this shard's scenes (camera split)

    @property
    def split(self) -> bool:
        return len(self.group_ranks) > 1


def plan(scenes: int, cameras: int, world: int) -> list[Shard]:
    """Placement of S scenes x C cameras on ``world`` ranks.

    world <= S: scene sharding (block partition), no collective.
    world > S:  ranks are grouped per scene (world must be a multiple of S and the
                group size at most C); each rank takes a camera block of its scene and
                the group all-reduces the scene's parameter gradients.
    """
    if world <= scenes:
        return [Shard(block(scenes, r, world), slice(0, cameras), (r,)) for r in range(world)]
    if world % scenes:
        raise ValueError(f"{world} ranks cannot split {scenes} scenes evenly")
    group = world // scenes
    if group > cameras:
        raise ValueError(f"{group} ranks per scene exceed its {cameras} cameras")
    shards = []
    for r in range(world):
        s, g = divmod(r, group)
        ranks = tuple(range(s * group, (s + 1) * group))
        shards.append(Shard(slice(s, s + 1), block(cameras, g, group), ranks))
    return shards


def take(inputs: dict, shard: Shard) -> dict:
    """This shard's slices of the public-API inputs (leading dims [S, ...])."""
    out = {}
    for name, t in inputs.items():
        part = t[shard.scenes]
        if name in PER_CAMERA:
            part = part[:, shard.cameras]
        out[name] = part.contiguous()
    return out


def allreduce_gradients(tensors, group=None) -> None:
    """Sum the ``.grad`` of ``tensors`` over ``group`` with one flattened bucket.

    Tensors without a gradient contribute zeros (every rank must take part in the
    same collective with the same bucket size).
    """
    tensors = list(tensors)
    if not tensors:
        return
    grads = [t.grad if t.grad is not None else torch.zeros_like(t) for t in tensors]
    bucket = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(bucket, op=dist.ReduceOp.SUM, group=group)
    offset = 0
    for t, g in zip(tensors, grads):
        n = g.numel()
        t.grad = bucket[offset:offset + n].view_as(g)
        offset += n


def groups_for(shards: list[Shard]):
    """Create one process group per distinct multi-rank gradient group (collective
    call: every rank must call it with the same plan, in the same order)."""
    made = {}
    for shard in shards:
        key = shard.group_ranks
        if len(key) > 1 and key not in made:
            made[key] = dist.new_group(list(key))
    return made
