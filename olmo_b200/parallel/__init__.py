"""Data-parallel execution: the flat-shard engine and its peer-memory collectives."""
from .fsdp import FlatShardEngine, ShardedModel, build_sharded_model

__all__ = ["FlatShardEngine", "ShardedModel", "build_sharded_model"]
