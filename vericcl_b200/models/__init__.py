"""Collective front ends (the "model families" of a collective library).

* :class:`CollectiveEngine` — AllReduce / AllGather / ReduceScatter on torch
  tensors with synthesized, verified schedules.
* :class:`GradBucketAllReduce` — data-parallel gradient buckets with a fused
  scale, one schedule replayed for every bucket.
"""
from .collectives import CollectiveEngine
from .grad_bucket import GradBucketAllReduce, DEFAULT_BUCKET_BYTES

__all__ = ["CollectiveEngine", "GradBucketAllReduce", "DEFAULT_BUCKET_BYTES"]
