"""Packed per-layer KV cache driven by liblrk operators.

The layout is the reference's flat cache contract (cache.py:16-265,
_core/cache.py:15-93): per layer, keys and values [rows, D] with the rows of
head 0, then head 1, ...; float32 position rows [rows, 1]; per-head lengths
on the host and cumulative lengths (int32) on the device.  This class is the
GPU branch of LazyRecallCache reduced to the KV bookkeeping: append
(cache.py:33-52 -> _C.append), remove_positions / remove_selected
(cache.py:92-180 -> _C.compact_layers), insert_payload (cache.py:201-253 ->
_C.merge_layers) and archive packing (recall/transport.py:148-167 ->
_C.pack).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Sequence, Tuple

import numpy as np

from . import operators, upload


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

    def spans(self):
        """(first row, end row) of each head in the layer tensors."""
        bounds = self.bounds().tolist()
        return list(zip(bounds[:-1], bounds[1:]))


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

        layer.cumulative = upload(layer.bounds().astype(np.int32), layer.keys.device)

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

    def segment_table(self, coordinates: Sequence[Tuple[int, int]]):
        """Per (layer, head) segment, as int64 [4, segments] on the device: the
        layer, the head's first row in the layer, its prompt rows and its rows."""
        import torch

        coordinates = np.asarray(coordinates, dtype=np.int64).reshape(-1, 2)
        used = np.unique(coordinates[:, 0])
        lens = np.asarray([self.layers[int(l)].head_lens for l in used], dtype=np.int64)
        prompts = np.asarray([self.layers[int(l)].prompt_lens for l in used], dtype=np.int64)
        starts = np.cumsum(lens, axis=1) - lens
        row, head = np.searchsorted(used, coordinates[:, 0]), coordinates[:, 1]
        table = np.stack((coordinates[:, 0], starts[row, head], prompts[row, head], lens[row, head]))
        return upload(table, self.layers[0].keys.device)

    def remove_selected(self, coordinates: Sequence[Tuple[int, int]], segment_ids, positions, table=None) -> int:
        """remove_positions for references that are still on the device:
        ``segment_ids`` and ``positions`` (int64 CUDA tensors, one entry per
        reference) index ``coordinates``.  The absolute rows are formed and
        sorted on the device; only per-segment counts (and two check counters)
        come back before the compactions are queued, so the device idles for
        the host bookkeeping alone.  A position outside its head raises
        IndexError before the cache changes; duplicate references fall back to
        remove_positions, which counts them once."""
        import torch

        if segment_ids.numel() == 0:
            return 0
        segments = len(coordinates)
        table = self.segment_table(coordinates) if table is None else table
        seg, pos = segment_ids.reshape(-1), positions.reshape(-1)
        layer_of, start, prompt, length = table[0][seg], table[1][seg], table[2][seg], table[3][seg]
        outside = ((pos < 0) | (pos >= length)).sum()
        keys = torch.sort(layer_of * (1 << 40) + start + pos).values
        duplicates = (keys[1:] == keys[:-1]).sum()
        # Counts by scatter-add (torch.bincount reads its input's maximum back
        # to the host first).
        counts = torch.zeros(2 * segments + 2, dtype=torch.int64, device=seg.device)
        counts.scatter_add_(0, seg, torch.ones_like(seg))
        counts.scatter_add_(0, seg + segments, (pos < prompt).to(torch.int64))
        counts[2 * segments] = outside
        counts[2 * segments + 1] = duplicates
        host = torch.empty(counts.shape, dtype=counts.dtype, pin_memory=True)
        host.copy_(counts, non_blocking=True)
        ready = torch.cuda.Event()
        ready.record()
        rows = keys & ((1 << 40) - 1)  # queued before the host waits
        ready.synchronize()
        counts = host.numpy()
        if counts[2 * segments]:
            first = int(torch.nonzero((pos < 0) | (pos >= length))[0, 0])
            layer_index, head = coordinates[int(seg[first])]
            raise IndexError(f"Invalid removal in layer={int(layer_index)}, head={int(head)}")
        if counts[2 * segments + 1]:
            return self.remove_positions({tuple(coordinates[s]): positions[seg == s].cpu().numpy()
                                          for s in np.flatnonzero(counts[:segments]).tolist()})
        per_layer = np.zeros(len(self.layers), dtype=np.int64)
        removed_counts, prompt_counts = counts[:segments], counts[segments:2 * segments]
        for s in np.flatnonzero(removed_counts).tolist():
            layer_index, head = coordinates[s]
            self.layers[layer_index].head_lens[head] -= int(removed_counts[s])
            self.layers[layer_index].prompt_lens[head] -= int(prompt_counts[s])
            per_layer[layer_index] += removed_counts[s]
        touched = np.flatnonzero(per_layer)
        offsets = np.concatenate(([0], np.cumsum(per_layer[touched]))).tolist()
        lens = np.asarray([self.layers[int(l)].head_lens for l in touched], dtype=np.int64)
        cumulative = np.zeros((touched.size, lens.shape[1] + 1), dtype=np.int32)
        np.cumsum(lens, axis=1, out=cumulative[:, 1:])
        all_cumulative = upload(cumulative, rows.device)
        layers = [self.layers[int(l)] for l in touched]
        keys_out, values_out, positions_out = operators().compact_layers(
            [layer.keys for layer in layers], [layer.values for layer in layers],
            [layer.positions for layer in layers], rows, offsets)
        for i, layer in enumerate(layers):
            layer.keys, layer.values, layer.positions = keys_out[i], values_out[i], positions_out[i]
            layer.cumulative = all_cumulative[i]
        return int(offsets[-1])

    def insert_payload(self, payload, metadata, plan: str = "device") -> int:
        """Recall reinsertion (cache.py:201-253): payload [n, 2, D] (K, V rows
        on the cache's device), metadata [n, 3] of (layer, head, position).
        Every touched head's rows are merged with its recalled rows in
        ascending position order (recall/planning.py:34-52).  The recalled
        rows are sorted by (layer, head, position) on the host and travel in
        one copy; the merge maps of all touched layers are planned on the
        device (lrk_merge_plan) from the resident positions, which never come
        to the host, and all touched layers move in one lrk_merge_layers
        launch (both through _C.reinsert_layers).  One flag word comes back before the merged tensors are
        adopted: a duplicate identity raises ValueError with the cache
        unchanged, and a head whose resident positions do not ascend (only a
        caller's own add_layer can make one) is re-planned on the host.
        ``plan="host"`` plans every layer on the host instead (the
        reference's numpy plan after one copy of the positions).  Returns the
        number of rows inserted."""
        import torch

        metadata = np.asarray(metadata, dtype=np.int64).reshape(-1, 3)
        if payload.shape[:2] != (len(metadata), 2):
            raise ValueError("Recall payload/identity shape mismatch")
        if plan not in ("device", "host"):
            raise ValueError(f"unknown merge plan {plan!r}")
        if not len(metadata):
            return 0
        touched = np.unique(metadata[:, 0]).tolist()
        layers = [self.layers[l] for l in touched]
        heads = len(layers[0].head_lens)
        if ((metadata[:, 1] < 0) | (metadata[:, 1] >= heads)).any():
            # The reference plans no row for such an identity and fails its
            # slot-count check after the merge; here the cache stays unchanged.
            raise AssertionError("Recall changed logical time or inserted an incorrect slot count")
        device = layers[0].keys.device
        order = np.lexsort((metadata[:, 2], metadata[:, 1], metadata[:, 0]))
        ordered = metadata[order]
        slot = np.searchsorted(touched, ordered[:, 0])  # each row's place among the touched layers
        firsts = np.searchsorted(slot, np.arange(len(layers) + 1))
        # Per touched layer, each head's first recalled row relative to the layer's first.
        starts = np.searchsorted(slot * heads + ordered[:, 1], np.arange(len(layers) * (heads + 1)) -
                                 np.repeat(np.arange(len(layers)), heads + 1)).reshape(len(layers), heads + 1)
        starts = (starts - firsts[:-1, None]).astype(np.int32)
        lens = np.asarray([layer.head_lens for layer in layers], dtype=np.int32)
        new_lens = lens + np.diff(starts, axis=1)
        bounds = np.zeros_like(starts)
        np.cumsum(new_lens, axis=1, out=bounds[:, 1:])
        # One upload: the payload rows in merge order, then the recalled starts
        # and new bounds (int32), then the positions (float32).
        int32_words = np.concatenate((starts.reshape(-1), bounds.reshape(-1)))
        int32_words = np.concatenate((int32_words, np.zeros(int32_words.size % 2, np.int32)))
        float_words = ordered[:, 2].astype(np.float32)
        float_words = np.concatenate((float_words, np.zeros(float_words.size % 2, np.float32)))
        words = upload(np.concatenate((order, int32_words.view(np.int64), float_words.view(np.int64))), device)
        n, table = len(order), starts.size
        small = words[n:n + int32_words.size // 2].view(torch.int32)
        positions = words[n + int32_words.size // 2:].view(torch.float32)[:n]
        all_bounds = small[table:2 * table].view(len(layers), heads + 1)
        recalled_rows = payload.index_select(0, words[:n]).contiguous()
        args = ([layer.keys for layer in layers], [layer.values for layer in layers],
                [layer.positions for layer in layers])
        if plan == "host":
            maps = self._host_merge_plan(layers, ordered, firsts)
            merged = operators().merge_layers(
                *args, [recalled_rows[firsts[i]:firsts[i + 1]] for i in range(len(layers))],
                [positions[firsts[i]:firsts[i + 1]] for i in range(len(layers))], [upload(m, device) for m in maps])
        else:
            *merged, flag = operators().reinsert_layers(
                *args, [layer.cumulative for layer in layers], recalled_rows, positions,
                small[:table], firsts.tolist())
            state = int(flag.item())
            if state & 4:
                raise RuntimeError("Cache head bounds do not match its rows")
            if state & 1:
                raise ValueError("Cannot merge duplicate physical KV identities")
            if state & 2:
                maps = self._host_merge_plan(layers, ordered, firsts)
                merged = operators().merge_layers(
                    *args, [recalled_rows[firsts[i]:firsts[i + 1]] for i in range(len(layers))],
                    [positions[firsts[i]:firsts[i + 1]] for i in range(len(layers))],
                    [upload(m, device) for m in maps])
        for i, layer in enumerate(layers):
            layer.keys, layer.values, layer.positions = merged[0][i], merged[1][i], merged[2][i]
            layer.head_lens = new_lens[i].tolist()
            layer.cumulative = all_bounds[i]
        return int(len(metadata))

    @staticmethod
    def _host_merge_plan(layers, ordered, firsts):
        """recall/planning.py:34-52 on the host (for heads whose resident
        positions do not ascend, or plan="host"): per head, the stable argsort of the resident
        positions followed by the recalled ones (``ordered``: the recalled
        identities sorted by layer, head, position; ``firsts``: each layer's
        first entry)."""
        import torch

        maps = []
        resident = torch.cat([layer.positions.reshape(-1) for layer in layers]).cpu().numpy().astype(np.int64)
        offsets = np.concatenate(([0], np.cumsum([sum(layer.head_lens) for layer in layers])))
        for i, layer in enumerate(layers):
            old = resident[offsets[i]:offsets[i + 1]]
            recalled = ordered[firsts[i]:firsts[i + 1]]
            mapping, start = [], 0
            for head, length in enumerate(layer.head_lens):
                chosen = np.flatnonzero(recalled[:, 1] == head)
                combined = np.concatenate((old[start:start + length], recalled[chosen, 2]))
                if np.unique(combined).size != combined.size:
                    raise ValueError("Cannot merge duplicate physical KV identities")
                sources = np.concatenate((np.arange(start, start + length), -chosen - 1))
                mapping.append(sources[np.argsort(combined, kind="stable")])
                start += length
            maps.append(np.concatenate(mapping))
        return maps

    def remove_positions(self, removals: Dict[Tuple[int, int], Sequence[int]]) -> int:
        """Drop head-relative rows (cache.py:92-180, GPU branch): one sorted
        absolute-row list, then one _C.compact_layers call (a compaction per
        touched layer).  Duplicate
        positions of a head count once; any position outside its head raises
        IndexError before the cache changes.  The host bookkeeping is
        vectorised over all (layer, head) entries, and the rows of every
        layer travel to the device in one copy."""
        import torch

        coordinates = np.asarray(list(removals.keys()), dtype=np.int64).reshape(-1, 2)
        arrays = [np.asarray(value, dtype=np.int64).reshape(-1) for value in removals.values()]
        sizes = np.asarray([a.size for a in arrays], dtype=np.int64)
        if not sizes.sum():
            return 0
        positions = np.concatenate(arrays)
        owner = np.repeat(np.arange(len(arrays)), sizes)
        order = np.lexsort((positions, owner))
        positions, owner = positions[order], owner[order]
        fresh = np.ones(positions.size, dtype=bool)
        fresh[1:] = (positions[1:] != positions[:-1]) | (owner[1:] != owner[:-1])
        positions, owner = positions[fresh], owner[fresh]
        bounds = {l: self.layers[l].bounds() for l in np.unique(coordinates[:, 0]).tolist()}
        head_lens = np.asarray([self.layers[l].head_lens[h] for l, h in coordinates.tolist()], dtype=np.int64)
        prompt_lens = np.asarray([self.layers[l].prompt_lens[h] for l, h in coordinates.tolist()], dtype=np.int64)
        bad = (positions < 0) | (positions >= head_lens[owner])
        if bad.any():
            layer_index, head = coordinates[owner[np.argmax(bad)]]
            raise IndexError(f"Invalid removal in layer={int(layer_index)}, head={int(head)}")
        starts = np.asarray([bounds[l][h] for l, h in coordinates.tolist()], dtype=np.int64)
        rows = starts[owner] + positions
        layer_of = coordinates[owner, 0]
        order = np.lexsort((rows, layer_of))
        rows, layer_of = rows[order], layer_of[order]
        removed = np.bincount(owner, minlength=len(arrays))
        removed_prompt = np.bincount(owner, weights=positions < prompt_lens[owner], minlength=len(arrays))
        for (layer_index, head), count, prompt in zip(coordinates.tolist(), removed.tolist(), removed_prompt.tolist()):
            self.layers[layer_index].head_lens[head] -= int(count)
            self.layers[layer_index].prompt_lens[head] -= int(prompt)
        touched, first = np.unique(layer_of, return_index=True)
        device = self.layers[int(touched[0])].keys.device
        all_rows = upload(rows, device)
        cumulative = np.stack([self.layers[int(l)].bounds() for l in touched]).astype(np.int32)
        all_cumulative = upload(cumulative, device)
        layers = [self.layers[int(l)] for l in touched]
        offsets = np.append(first, rows.size).tolist()
        keys, values, positions = operators().compact_layers(
            [layer.keys for layer in layers], [layer.values for layer in layers],
            [layer.positions for layer in layers], all_rows, offsets)
        for i, layer in enumerate(layers):
            layer.keys, layer.values, layer.positions = keys[i], values[i], positions[i]
            layer.cumulative = all_cumulative[i]
        return int(removed.sum())
