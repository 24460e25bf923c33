"""Camera -> GPU partition for multi-GPU runs: a frame stays on the GPU that holds it.

Restates the camera assignment of the reference's ``plan_shards``
(``src/shipinfer/scheduling/sharding.py:200-300``) for the case this package runs, one shard
per GPU: longest-processing-time-first over offered fps, ties broken by camera id, each camera
going to the shard with the least load per unit of device. The GPUs never exchange pixels, so
there is no collective on the data path; ranks only agree on this plan.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence

from shipinfer_b200.errors import ConfigurationError

__all__ = ["plan_cameras", "shard_of"]


def plan_cameras(load: Mapping[str, float], gpus: Sequence[int]) -> list[tuple[str, ...]]:
    """Cameras per GPU (index-aligned with ``gpus``), each tuple sorted by camera id.

    Raises:
        ConfigurationError: no GPUs, or more GPUs than cameras (a GPU with no camera would
            hold a context and read nothing — the reference refuses it for the same reason).
    """
    shards = len(gpus)
    if shards < 1:
        raise ConfigurationError("cannot plan shards with no gpus")
    if load and shards > len(load):
        raise ConfigurationError(f"{shards} GPUs for {len(load)} camera(s); use at most {len(load)}")
    buckets: list[list[str]] = [[] for _ in range(shards)]
    weights = [0.0] * shards
    for name in sorted(load, key=lambda n: (-load[n], n)):
        target = min(range(shards), key=lambda i: (weights[i], i))
        buckets[target].append(name)
        weights[target] += load[name]
    return [tuple(sorted(b)) for b in buckets]


def shard_of(load: Mapping[str, float], gpus: Sequence[int], rank: int) -> tuple[str, ...]:
    """The cameras rank ``rank`` owns under :func:`plan_cameras` (every rank computes the same
    plan independently; nothing is communicated)."""
    return plan_cameras(load, gpus)[rank]
