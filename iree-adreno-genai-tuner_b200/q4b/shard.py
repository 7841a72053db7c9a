"""Tensor-parallel shards of one packed int4 linear (qweight [N, K/8] int32, scales [N, K/G] fp16),
for a projection sharded on its own (BASELINE config 5 across GPUs; the model's layers shard before
quantisation, q4b.shard_layer).

  split "col"  rank r holds output rows [r N/t, (r+1) N/t): y_r = x W_r^T, no collective (the
               outputs concatenate in rank order)
  split "row"  rank r holds the k columns [r K/t, (r+1) K/t) and the matching x columns: the ranks'
               partial outputs sum to y (an all-reduce)

Pure tensor slicing on whatever device the inputs live on."""

from __future__ import annotations


def shard_ok(n: int, k: int, group: int, world: int, split: str) -> bool:
    """Whether the split keeps every shard on whole rows (col) or whole scale groups (row)."""
    if split == "col":
        return n % world == 0
    if split == "row":
        return k % world == 0 and (k // world) % group == 0
    raise ValueError(f"split must be 'col' or 'row', not {split!r}")


def shard_q4(qweight, scales, group: int, rank: int, world: int, split: str):
    """(qweight, scales) of rank `rank` of `world` (contiguous copies)."""
    n, k = qweight.shape[0], qweight.shape[1] * 8
    if not shard_ok(n, k, group, world, split):
        raise ValueError(f"{n}x{k} (group {group}) does not split {split}-wise over {world} ranks")
    if split == "col":
        r0, r1 = rank * n // world, (rank + 1) * n // world
        return qweight[r0:r1].contiguous(), scales[r0:r1].contiguous()
    k0, k1 = rank * k // world, (rank + 1) * k // world
    return qweight[:, k0 // 8:k1 // 8].contiguous(), scales[:, k0 // group:k1 // group].contiguous()


def shard_x(x, rank: int, world: int, split: str):
    """The x [M, K] columns rank `rank` multiplies: all of x (col), or its k slice (row)."""
    if split == "col":
        return x
    k = x.shape[1]
    return x[:, rank * k // world:(rank + 1) * k // world].contiguous()
