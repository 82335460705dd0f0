"""Row partition for one-process-per-GPU sharding (used by bench.py and the sharded tests).

Rank r of `world` owns rows [r*n//world, (r+1)*n//world): contiguous shards whose sizes differ by
at most one row, with global ids = shard offset + local id, so the cross-shard merge by
(distance, global id) reproduces the single-index order exactly."""


def row_range(rank: int, world: int, n: int) -> tuple[int, int]:
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    return rank * n // world, (rank + 1) * n // world
