"""Writes a ``torch_legacy`` style sharded checkpoint (``rank{r}.pt`` with real ``ShardedTensor`` objects, chunked along
dimension 0 the way FSDP1's sharded state dict chunks them) from known full tensors.  Runs as gloo ranks on CPU."""
import argparse
import math
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist
from torch.distributed._shard.sharded_tensor import Shard, ShardMetadata, init_from_local_shards

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def to_sharded(full: torch.Tensor, rank: int, world: int):
    rows = full.shape[0]
    chunk = math.ceil(rows / world)
    lo, hi = min(rank * chunk, rows), min((rank + 1) * chunk, rows)
    shards = []
    if hi > lo:
        offsets = [lo] + [0] * (full.dim() - 1)
        sizes = [hi - lo] + list(full.shape[1:])
        shards.append(Shard(full[lo:hi].clone(), ShardMetadata(shard_offsets=offsets, shard_sizes=sizes, placement=f"rank:{rank}/cpu")))
    return init_from_local_shards(shards, *full.shape)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--source", required=True, help="torch file with {'model': {...}, 'optim': {...}, 'trainer': {...}} full tensors")
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    dist.init_process_group("gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    src = torch.load(args.source, weights_only=False)
    model = {f"transformer.{k}" if False else k: to_sharded(v, rank, world) for k, v in src["model"].items()}
    optim_state = {}
    for name, entries in src["optim"]["state"].items():
        optim_state[name] = {k: (to_sharded(v, rank, world) if isinstance(v, torch.Tensor) and v.dim() > 0 else v) for k, v in entries.items()}
    state = {"model": model, "optim": {"state": optim_state, "param_groups": src["optim"]["param_groups"]}, **src["trainer"]}
    os.makedirs(args.out, exist_ok=True)
    torch.save(state, Path(args.out) / f"rank{rank}.pt")
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
