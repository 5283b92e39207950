"""Packed per-layer KV cache driven by liblrk operators.

The layout is the reference's flat cache contract (cache.py:16-265,
_core/cache.py:15-93): per layer, keys and values [rows, D] with the rows of
head 0, then head 1, ...; float32 position rows [rows, 1]; per-head lengths
on the host and cumulative lengths (int32) on the device.  This class is the
GPU branch of LazyRecallCache reduced to the KV bookkeeping: append
(cache.py:33-52 -> _C.append), remove_positions (cache.py:92-180 ->
_C.compact), insert_payload (cache.py:201-253 -> _C.merge) and archive
packing (recall/transport.py:148-167 -> _C.pack).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Sequence, Tuple

import numpy as np

from . import operators


@dataclass
class LayerState:
    keys: "object"
    values: "object"
    positions: "object"
    head_lens: List[int]
    prompt_lens: List[int]
    cumulative: "object" = None  # int32 [heads + 1] on the device

    def bounds(self) -> np.ndarray:
        return np.concatenate(([0], np.cumsum(self.head_lens))).astype(np.int64)


@dataclass
class PackedCache:
    layers: List[LayerState] = field(default_factory=list)
    seen_tokens: int = 0

    @property
    def heads(self) -> int:
        return len(self.layers[0].head_lens)

    def total_rows(self) -> int:
        return sum(sum(layer.head_lens) for layer in self.layers)

    def generation_rows(self) -> int:
        return sum(sum(layer.head_lens) - sum(layer.prompt_lens) for layer in self.layers)

    def _refresh(self, layer: LayerState) -> None:
        import torch

        layer.cumulative = torch.as_tensor(layer.bounds(), dtype=torch.int32).to(layer.keys.device,
                                                                                  non_blocking=True)

    def add_layer(self, keys, values, positions, head_lens: Sequence[int], prompt_lens: Sequence[int]) -> None:
        state = LayerState(keys, values, positions.reshape(-1, 1), list(map(int, head_lens)),
                           list(map(int, prompt_lens)))
        self._refresh(state)
        self.layers.append(state)

    def append(self, layer_index: int, new_keys, new_values, logical_start: int) -> None:
        """One decode step for one layer (cache.py:33-52): new_* [1, H, 1, D]."""
        layer = self.layers[layer_index]
        keys, values, positions, cumulative, _ = operators().append(
            layer.keys, layer.values, layer.positions, new_keys, new_values, layer.cumulative, logical_start,
            max(layer.head_lens))
        added = new_keys.shape[2]
        layer.keys, layer.values, layer.positions, layer.cumulative = keys, values, positions, cumulative
        layer.head_lens = [length + added for length in layer.head_lens]

    def remove_positions(self, removals: Dict[Tuple[int, int], Sequence[int]]) -> int:
        """Drop head-relative rows (cache.py:92-180, GPU branch): one sorted
        absolute-row list and one _C.compact per touched layer."""
        import torch

        grouped: Dict[int, Dict[int, np.ndarray]] = {}
        for (layer_index, head), positions in removals.items():
            positions = np.unique(np.asarray(positions, dtype=np.int64))
            if positions.size:
                grouped.setdefault(layer_index, {})[head] = positions
        by_layer: Dict[int, List[np.ndarray]] = {}
        removed_total = 0
        for layer_index, heads in grouped.items():
            layer = self.layers[layer_index]
            bounds = layer.bounds()
            for head, positions in heads.items():
                if positions[0] < 0 or positions[-1] >= layer.head_lens[head]:
                    raise IndexError(f"Invalid removal in layer={layer_index}, head={head}")
                by_layer.setdefault(layer_index, []).append(bounds[head] + positions)
            for head, positions in heads.items():
                layer.head_lens[head] -= int(positions.size)
                layer.prompt_lens[head] -= int(np.sum(positions < layer.prompt_lens[head]))
                removed_total += int(positions.size)
        for layer_index, parts in by_layer.items():
            layer = self.layers[layer_index]
            ordered = torch.as_tensor(np.sort(np.concatenate(parts)), dtype=torch.int64).to(layer.keys.device,
                                                                                             non_blocking=True)
            layer.keys, layer.values, layer.positions = operators().compact(layer.keys, layer.values,
                                                                            layer.positions, ordered)
            self._refresh(layer)
        return removed_total
