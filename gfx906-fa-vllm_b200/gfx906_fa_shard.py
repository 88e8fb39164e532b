"""Head sharding of the attention path across tensor-parallel ranks.

Attention needs no exchange between ranks: vLLM's tensor parallelism gives
each rank a contiguous group of query heads and the kv heads they read, and
each rank's KV cache holds only those kv heads.  When there are more ranks
than kv heads, vLLM replicates each kv head over world / num_heads_kv ranks
(vllm/model_executor/layers/linear.py QKVParallelLinear: num_kv_head_replicas).
"""
from dataclasses import dataclass


@dataclass(frozen=True)
class HeadShard:
    q0: int          # first query head of this rank
    q1: int          # one past the last
    kv0: int         # first kv head of this rank
    kv1: int         # one past the last

    @property
    def num_heads_q(self) -> int:
        return self.q1 - self.q0

    @property
    def num_heads_kv(self) -> int:
        return self.kv1 - self.kv0


def head_shard(num_heads_q: int, num_heads_kv: int, world: int, rank: int) -> HeadShard:
    """Query / kv head ranges owned by `rank` of `world`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if num_heads_q % world:
        raise ValueError(f"{num_heads_q} query heads do not split over {world} ranks")
    if num_heads_q % num_heads_kv:
        raise ValueError("query heads must be a multiple of kv heads")
    qn = num_heads_q // world
    if world <= num_heads_kv:
        if num_heads_kv % world:
            raise ValueError(f"{num_heads_kv} kv heads do not split over {world} ranks")
        kn = num_heads_kv // world
        return HeadShard(rank * qn, (rank + 1) * qn, rank * kn, (rank + 1) * kn)
    if world % num_heads_kv:
        raise ValueError(f"{world} ranks do not replicate {num_heads_kv} kv heads evenly")
    kv = rank // (world // num_heads_kv)
    return HeadShard(rank * qn, (rank + 1) * qn, kv, kv + 1)
