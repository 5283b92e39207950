"""Drop-in replacement for LazyRecall's selection step on the GPU.

refine_arrays(allocation, refinement, count) keeps the signature, checks and
return value of selection.py:52-88 in the reference: a rank-slot queue
(ArrayReferences) plus the number of changed identities and changed heads.
The body -- global bottom-`count` of raw scores, per-head quotas, per-head
bottom-quota of pooled scores and the transplant of those picks into the
raw-score slots -- runs as one sequence of liblrk kernels (_C.refine) with a
single device-to-host copy of the finished queue at the end.  Tie handling
reproduces torch.topk(largest=False, sorted=True) on CUDA, which is what the
reference calls.

Integration: a caller that wants the reference's own ArrayReferences class
passes it as ``references_type``; by default the equivalent class below is
returned.
"""
from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import numpy as np

from . import operators, upload


@dataclass(order=True, frozen=True)
class KVReference:
    """One queued identity: its raw score, layer, KV head and head-local row."""
    score: float
    layer: int
    head: int
    position: int


class ArrayReferences(Sequence):
    """Column-store queue of KV identities in eviction order.

    Same interface as the reference's queue type: ``scores``, ``segments``,
    ``positions`` (one entry per queue slot), ``coordinates`` (segment ->
    (layer, head)), slicing, item access as :class:`KVReference` and
    :meth:`groups` ((layer, head) -> sorted positions)."""

    def __init__(self, scores, segments, positions, coordinates):
        self.scores = np.asarray(scores)
        self.segments = np.asarray(segments, dtype=np.int64)
        self.positions = np.asarray(positions, dtype=np.int64)
        self.coordinates = np.asarray(coordinates, dtype=np.int64).reshape(-1, 2)
        if not len(self.scores) == len(self.segments) == len(self.positions):
            raise ValueError("Queue column lengths differ")

    def __len__(self):
        return int(self.positions.shape[0])

    def __getitem__(self, index):
        if isinstance(index, slice):
            return type(self)(self.scores[index], self.segments[index], self.positions[index], self.coordinates)
        layer, head = self.coordinates[self.segments[index]]
        return KVReference(float(self.scores[index]), int(layer), int(head), int(self.positions[index]))

    def groups(self):
        """(layer, head) -> ascending positions queued for that head, in
        ascending segment order."""
        result = {}
        if not len(self):
            return result
        order = np.lexsort((self.positions, self.segments))
        segments, positions = self.segments[order], self.positions[order]
        cuts = np.flatnonzero(segments[1:] != segments[:-1]) + 1
        for segment, part in zip(segments[np.concatenate(([0], cuts))].tolist(), np.split(positions, cuts)):
            layer, head = self.coordinates[segment]
            result[(int(layer), int(head))] = part
        return result


def refine_arrays(allocation, refinement, count, references_type=None):
    """GPU refine_arrays (selection.py:52-88).  ``allocation`` and
    ``refinement`` are score tables with ``scores`` (1-D float32 CUDA tensor),
    ``segments`` (objects with layer, head, position_start, count) and
    ``cumulative_ends``.  Returns (references, changed, changed_heads)."""
    return fetch_references(refine_device(allocation, refinement, count), references_type).result()


@dataclass
class DeviceQueue:
    """refine_arrays' queue before it leaves the device: ``count`` slots of
    raw-score bits, segment ids and head-local positions (CUDA tensors), the
    two change counters, and the segment -> (layer, head) coordinates."""
    values: object
    segment_ids: object
    positions: object
    stats: object
    count: int
    coordinates: list


def refine_device(allocation, refinement, count) -> DeviceQueue:
    """refine_arrays up to its device-to-host copy: the same checks, then the
    _C.refine kernels.  Nothing waits for the device."""
    import torch

    if allocation.segments != refinement.segments or allocation.cumulative_ends != refinement.cumulative_ends:
        raise ValueError("Allocation and refinement layouts differ")
    coordinates = [(segment.layer, segment.head) for segment in allocation.segments]
    if len(set(coordinates)) != len(coordinates):
        raise ValueError("Each physical head must have exactly one score segment")
    count = min(max(0, int(count)), allocation.scores.numel())
    if not count:
        return DeviceQueue(None, None, None, None, 0, coordinates)
    ends = np.asarray(allocation.cumulative_ends, dtype=np.int64)
    starts = np.concatenate(([0], ends[:-1]))
    if ends[-1] != allocation.scores.numel() or any(
            end - start != segment.count for start, end, segment in zip(starts, ends, allocation.segments)):
        raise ValueError("Invalid segment bounds")
    raw = allocation.scores
    if not raw.is_cuda:
        raise RuntimeError("refine_arrays runs on CUDA score tables only")
    device = raw.device
    host = np.stack([ends, np.asarray([segment.position_start for segment in allocation.segments], dtype=np.int64)])
    ends_device, position_starts = upload(host, device)
    values, segment_ids, positions, stats = operators().refine(
        raw.float().contiguous(), refinement.scores.float().contiguous(), ends_device, position_starts, count)
    return DeviceQueue(values, segment_ids, positions, stats, count, coordinates)


class PendingReferences:
    """A queue on its way to the host: asynchronous device-to-host copies
    into pinned memory -- segment ids, positions and the two counters into one
    int64 buffer, the raw scores into a float32 buffer -- and the event after
    them.  result() waits for that event only, so work queued on the stream
    after the copies keeps the device busy meanwhile; the returned arrays are
    views of the pinned buffers (no conversion or copy on the host)."""

    def __init__(self, queue: DeviceQueue, references_type=None):
        import torch

        self.make = references_type or ArrayReferences
        self.queue = queue
        if not queue.count:
            return
        count = queue.count
        self.host = torch.empty(2 * count + 2, dtype=torch.int64, pin_memory=True)
        self.host[:count].copy_(queue.segment_ids, non_blocking=True)
        self.host[count:2 * count].copy_(queue.positions, non_blocking=True)
        self.host[2 * count:].copy_(queue.stats, non_blocking=True)
        self.host_values = torch.empty(count, dtype=torch.float32, pin_memory=True)
        self.host_values.copy_(queue.values, non_blocking=True)
        self.event = torch.cuda.Event()
        self.event.record()

    def result(self):
        queue = self.queue
        if not queue.count:
            return self.make([], [], [], queue.coordinates), 0, 0
        self.event.synchronize()
        packed, count = self.host.numpy(), queue.count
        changed, changed_heads = int(packed[2 * count]), int(packed[2 * count + 1])
        return (self.make(self.host_values.numpy(), packed[:count], packed[count:2 * count], queue.coordinates),
                changed, changed_heads)


def fetch_references(queue: DeviceQueue, references_type=None) -> PendingReferences:
    return PendingReferences(queue, references_type)


def allocation_preserving_references(allocation_table, refinement_table, count, references_type=None):
    """scoring.py:356-361 without the timing wrapper: refine_arrays' result."""
    return refine_arrays(allocation_table, refinement_table, count, references_type)
