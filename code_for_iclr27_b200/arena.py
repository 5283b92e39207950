"""Gapped per-head KV arena: decode appends and evictions without whole-layer copies.

The reference's cache (cache.py:16-265) keeps each layer packed -- K, V
[rows, D] with the heads back to back -- and replaces the layer's tensors on
every append (cache.py:33-52), compaction (cache.py:157-170) and merge
(cache.py:240-246), so every decode step moves every layer through HBM
(1.8 ms per step at configs[1]).  ArenaCache gives each (layer, head) a slot
of `capacity` rows in three tensors for the whole cache -- keys and values
[layers * heads, capacity, D], positions [layers * heads, capacity] -- with the
head lengths on the device (int32) and mirrored on the host:

* append_all: one lrk_arena_append launch writes one row per head of every
  layer (2 D + 4 bytes per head) and advances the lengths;
* remove_positions / remove_selected: one lrk_arena_compact launch shifts
  the rows after each touched head's first removed row down, in place; heads
  without removals do not move.

A head's live rows are rows [0, length) of its slot, in the packed layout's
order, so the packed layer is the slots' live rows back to back (packed_layer;
the tests check both caches bit for bit through the same operations).  The
scoring path reads the arena as it is: each layer view is keys/values
[heads * capacity, D] with head h at rows [h * capacity, h * capacity +
length), which lrk_logits_heads, lrk_project_values and lrk_temporal_scores
take as spans.  FlashAttention reads it as flash_attn_with_kvcache(q [heads, 1,
G, D], k_cache=keys[layer] viewed [heads, capacity, 1, D], v_cache, cache_seqlens
= the layer's lengths), the decode counterpart of the reference's
flash_attn_varlen_func call on the packed layer (attention.py:15-35).

The class exposes what audit_pass, evict_prefix and a decode loop use of
PackedCache (layers, segment_table, remove_selected, remove_positions,
append), so the audit runs on it unchanged.
"""
from __future__ import annotations

from typing import Dict, List, Sequence, Tuple

import numpy as np

from . import operators, upload


class ArenaLayer:
    """One layer of an ArenaCache, shaped like kvcache.LayerState: keys and
    values [heads * capacity, D], positions [heads * capacity, 1] (views of the
    arena), the host head/prompt lengths, and `cumulative` = the slot starts
    (int32 [heads + 1], device), which assigns every arena row to its head for
    lrk_project_values."""

    def __init__(self, cache: "ArenaCache", index: int):
        heads, cap = cache.heads, cache.capacity
        rows = slice(index * heads, (index + 1) * heads)
        self.keys = cache.keys[rows].view(heads * cap, -1)
        self.values = cache.values[rows].view(heads * cap, -1)
        self.positions = cache.positions[rows].view(heads * cap, 1)
        self.head_lens = cache.head_lens[index]
        self.prompt_lens = cache.prompt_lens[index]
        self.cumulative = cache.slot_starts
        self.capacity = cap

    def spans(self) -> List[Tuple[int, int]]:
        """(first row, end row) of each head's live rows in the layer views."""
        return [(h * self.capacity, h * self.capacity + n) for h, n in enumerate(self.head_lens)]


class ArenaCache:
    def __init__(self, layers: int, heads: int, dim: int, capacity: int, device, dtype=None):
        import torch

        dtype = dtype or torch.bfloat16
        self.heads, self.dim, self.capacity, self.device = heads, dim, int(capacity), torch.device(device)
        self.keys = torch.empty(layers * heads, self.capacity, dim, dtype=dtype, device=self.device)
        self.values = torch.empty_like(self.keys)
        self.positions = torch.zeros(layers * heads, self.capacity, dtype=torch.float32, device=self.device)
        self.lengths = torch.zeros(layers * heads, dtype=torch.int32, device=self.device)
        # Host mirrors [layers, heads]: exact, except after evict_logical
        # (device-only evictions), which leaves the live lengths on the device
        # until the next read here (_sync).
        self._head_lens = np.zeros((layers, heads), dtype=np.int64)
        self.prompt_lens = np.zeros((layers, heads), dtype=np.int64)
        self._stale = False
        self.seen_tokens = 0
        # Device flags the kernels set on a full slot or a bad removal list
        # (checked by callers that want to: check_flags).
        self.flags = torch.zeros(2, dtype=torch.int32, device=self.device)
        self._slot_starts()

    @property
    def head_lens(self) -> np.ndarray:
        """Live rows per [layer, head] (numpy; rows are views)."""
        self._sync()
        return self._head_lens

    def _sync(self) -> None:
        if self._stale:
            self._stale = False
            self._head_lens[:] = self.lengths.cpu().numpy().reshape(self._head_lens.shape)

    def _slot_starts(self):
        import torch

        self.slot_starts = torch.arange(0, (self.heads + 1) * self.capacity, self.capacity, dtype=torch.int32,
                                        device=self.device)

    # ------------------------------------------------------------ building

    @classmethod
    def from_packed(cls, packed, margin: int = 512) -> "ArenaCache":
        """An arena holding the same rows as a kvcache.PackedCache, each slot
        `margin` rows longer than the longest head."""
        import torch

        first = packed.layers[0]
        heads, dim = len(first.head_lens), first.keys.shape[-1]
        longest = max(max(layer.head_lens) for layer in packed.layers)
        arena = cls(len(packed.layers), heads, dim, longest + margin, first.keys.device, first.keys.dtype)
        for l, layer in enumerate(packed.layers):
            bounds = layer.bounds()
            for h in range(heads):
                a, b = int(bounds[h]), int(bounds[h + 1])
                arena.keys[l * heads + h, :b - a] = layer.keys[a:b]
                arena.values[l * heads + h, :b - a] = layer.values[a:b]
                arena.positions[l * heads + h, :b - a] = layer.positions.reshape(-1)[a:b]
            arena.head_lens[l] = layer.head_lens
            arena.prompt_lens[l] = layer.prompt_lens
        arena.lengths.copy_(torch.from_numpy(arena.head_lens.reshape(-1).astype(np.int32)))
        arena.seen_tokens = packed.seen_tokens
        return arena

    # --------------------------------------------------------------- views

    @property
    def layers(self) -> List[ArenaLayer]:
        return [ArenaLayer(self, l) for l in range(len(self.head_lens))]

    def total_rows(self) -> int:
        return int(self.head_lens.sum())

    def packed_layer(self, index: int):
        """The layer in the packed layout (K, V [rows, D], positions [rows, 1]):
        the heads' live rows back to back (a copy)."""
        import torch

        rows = torch.cat([torch.arange(n, device=self.device) + (index * self.heads + h) * self.capacity
                          for h, n in enumerate(self.head_lens[index])])
        flat_k = self.keys.view(-1, self.dim)
        flat_v = self.values.view(-1, self.dim)
        return (flat_k.index_select(0, rows), flat_v.index_select(0, rows),
                self.positions.view(-1).index_select(0, rows).view(-1, 1))

    def segment_table(self, coordinates: Sequence[Tuple[int, int]]):
        """As PackedCache.segment_table: int64 [4, segments] (layer, the head's
        first row in the layer view, prompt rows, rows) on the device."""
        coordinates = np.asarray(coordinates, dtype=np.int64).reshape(-1, 2)
        table = np.empty((4, coordinates.shape[0]), dtype=np.int64)
        for i, (l, h) in enumerate(coordinates.tolist()):
            table[:, i] = (l, h * self.capacity, self.prompt_lens[l][h], self.head_lens[l][h])
        return upload(table, self.device)

    # -------------------------------------------------------------- append

    def _grow(self, extra: int) -> None:
        """Reallocate every slot `extra` rows longer (rare: callers size the
        capacity for the run)."""
        import torch

        old = self.capacity
        self.capacity = old + int(extra)
        for name in ("keys", "values", "positions"):
            tensor = getattr(self, name)
            grown = torch.zeros((tensor.shape[0], self.capacity) + tuple(tensor.shape[2:]), dtype=tensor.dtype,
                                device=self.device)
            grown[:, :old] = tensor
            setattr(self, name, grown)
        self._slot_starts()

    def append_all(self, new_keys, new_values, logical_position: int) -> None:
        """One decode step for every layer in one launch: new_* [layers * heads,
        D] (or any shape with that many rows), all at `logical_position`
        (cache.py:33-52 gives every layer of a step the same position).  The
        capacity check uses the host mirror, an upper bound of the live
        lengths, so it needs no device round trip."""
        if int(self._head_lens.max()) >= self.capacity:
            self._sync()
            if int(self._head_lens.max()) >= self.capacity:
                self._grow(max(256, self.capacity // 8))
        operators().arena_append_into(self.keys, self.values, self.positions, self.lengths, 0,
                                      new_keys.reshape(-1, self.dim), new_values.reshape(-1, self.dim),
                                      float(logical_position), self.flags[0:1])
        self._head_lens += 1

    def append(self, layer_index: int, new_keys, new_values, logical_start: int) -> None:
        """One decode step for one layer (PackedCache.append's interface):
        new_* [1, heads, 1, D]."""
        if int(self.head_lens[layer_index].max()) >= self.capacity:
            self._grow(max(256, self.capacity // 8))
        operators().arena_append(self.keys, self.values, self.positions, self.lengths, layer_index * self.heads,
                                 new_keys.reshape(-1, self.dim), new_values.reshape(-1, self.dim),
                                 float(logical_start))
        self._head_lens[layer_index] += 1

    # ------------------------------------------------------------ eviction

    def _compact(self, flat_heads: np.ndarray, counts: np.ndarray, removed) -> None:
        """lrk_arena_compact over distinct heads (ascending), removed rows
        grouped by head in that order (a device int64 tensor)."""
        offsets = np.concatenate(([0], np.cumsum(counts)[:-1])).astype(np.int64)
        plan = upload(np.stack([flat_heads, offsets, counts], axis=1).astype(np.int64), self.device)
        operators().arena_compact(self.keys, self.values, self.positions, self.lengths, plan, removed)

    def remove_positions(self, removals: Dict[Tuple[int, int], Sequence[int]]) -> int:
        """Drop head-relative rows (cache.py:92-180): duplicates count once,
        any position outside its head raises IndexError before the cache
        changes.  One in-place compaction launch for every touched head."""
        entries = []
        for (layer, head), positions in removals.items():
            rows = np.unique(np.asarray(positions, dtype=np.int64).reshape(-1))
            if not rows.size:
                continue
            if rows[0] < 0 or rows[-1] >= self.head_lens[layer][head]:
                raise IndexError(f"Invalid removal in layer={int(layer)}, head={int(head)}")
            entries.append((int(layer) * self.heads + int(head), int(layer), int(head), rows))
        if not entries:
            return 0
        entries.sort(key=lambda e: e[0])
        lens = self.head_lens
        for _, layer, head, rows in entries:
            lens[layer][head] -= int(rows.size)
            self.prompt_lens[layer][head] -= int((rows < self.prompt_lens[layer][head]).sum())
        removed = upload(np.concatenate([e[3] for e in entries]), self.device)
        counts = np.asarray([e[3].size for e in entries], dtype=np.int64)
        self._compact(np.asarray([e[0] for e in entries], dtype=np.int64), counts, removed)
        return int(counts.sum())

    def remove_selected(self, coordinates: Sequence[Tuple[int, int]], segment_ids, positions, table=None) -> int:
        """remove_positions for references still on the device (as
        PackedCache.remove_selected): the rows are keyed (flat head, position)
        and sorted on the device; per-segment counts and two check counters
        come back before the compaction is queued."""
        import torch

        if segment_ids.numel() == 0:
            return 0
        segments = len(coordinates)
        table = self.segment_table(coordinates) if table is None else table
        seg, pos = segment_ids.reshape(-1), positions.reshape(-1)
        flat = table[0][seg] * self.heads + table[1][seg] // self.capacity
        prompt, length = table[2][seg], table[3][seg]
        outside = ((pos < 0) | (pos >= length)).sum()
        keys = torch.sort(flat * (1 << 32) + pos).values
        duplicates = (keys[1:] == keys[:-1]).sum()
        counts = torch.zeros(2 * segments + 2, dtype=torch.int64, device=seg.device)
        counts.scatter_add_(0, seg, torch.ones_like(seg))
        counts.scatter_add_(0, seg + segments, (pos < prompt).to(torch.int64))
        counts[2 * segments] = outside
        counts[2 * segments + 1] = duplicates
        host = torch.empty(counts.shape, dtype=counts.dtype, pin_memory=True)
        host.copy_(counts, non_blocking=True)
        ready = torch.cuda.Event()
        ready.record()
        removed = keys & ((1 << 32) - 1)
        ready.synchronize()
        counts = host.numpy()
        if counts[2 * segments]:
            first = int(torch.nonzero((pos < 0) | (pos >= length))[0, 0])
            layer_index, head = coordinates[int(seg[first])]
            raise IndexError(f"Invalid removal in layer={int(layer_index)}, head={int(head)}")
        if counts[2 * segments + 1]:
            return self.remove_positions({tuple(coordinates[s]): positions[seg == s].cpu().numpy()
                                          for s in np.flatnonzero(counts[:segments]).tolist()})
        touched = np.flatnonzero(counts[:segments])
        coords = np.asarray(coordinates, dtype=np.int64).reshape(-1, 2)[touched]
        flat_heads = coords[:, 0] * self.heads + coords[:, 1]
        order = np.argsort(flat_heads)
        lens = self.head_lens
        for s, (layer, head) in zip(touched.tolist(), coords.tolist()):
            lens[layer][head] -= int(counts[s])
            self.prompt_lens[layer][head] -= int(counts[segments + s])
        self._compact(flat_heads[order], counts[:segments][touched][order], removed)
        return int(counts[:segments].sum())

    # ------------------------------------------ lazy eviction on the device

    def queue_positions(self, table, segment_ids, positions):
        """Each queued reference's (flat head, logical position), gathered on
        the device from the rows it names now (call before those rows move):
        a lazy batch later finds each reference's current row from them alone
        (evict_logical)."""
        seg, pos = segment_ids.reshape(-1), positions.reshape(-1)
        flat = table[0][seg] * self.heads + table[1][seg] // self.capacity
        logical = self.positions.view(-1).index_select(0, flat * self.capacity + pos)
        return flat, logical

    def evict_logical(self, flat_heads, logical) -> None:
        """Lazy eviction of a batch of queued references (controller.py:57-70)
        with no host round trip: the references (flat head, logical position;
        queue_positions) go to one lrk_arena_evict launch, in which each head
        collects and sorts its own entries, finds their rows by position and
        shifts its rows in place.  The host length mirror becomes an upper
        bound until it is next read."""
        if flat_heads.numel() == 0:
            return
        operators().arena_evict(self.keys, self.values, self.positions, self.lengths, flat_heads.contiguous(),
                                logical.contiguous(), self.flags[1:2])
        self._stale = True

    # -------------------------------------------------------------- recall

    # Entries one lrk_arena_insert launch takes per head; a larger event goes
    # in rounds (merging in rounds gives the same rows: the order is by position).
    INSERT_MAX = 2048

    def insert_payload(self, payload, metadata) -> int:
        """Recall reinsertion in place (cache.py:201-253): payload [n, 2, D]
        (K, V rows on the arena's device), metadata [n, 3] of (layer, head,
        position).  Each touched head's rows above its first recalled
        position move up inside its slot and the recalled rows land in
        position order -- the rows and positions the reference's merge gives
        the head -- with no layer copied.  A check launch runs first and its
        flag is read before anything moves: a position recalled twice or
        recalled while resident raises ValueError (cache unchanged, as the
        reference refuses the merge); a head whose positions do not ascend
        raises ValueError too (the arena keeps heads in position order; a
        caller-built arena may not).  A head without room grows every slot
        first.  Returns the number of rows inserted."""
        import torch

        metadata = np.asarray(metadata, dtype=np.int64).reshape(-1, 3)
        if payload.shape[:2] != (len(metadata), 2):
            raise ValueError("Recall payload/identity shape mismatch")
        if not len(metadata):
            return 0
        layers = len(self.head_lens)
        if ((metadata[:, 1] < 0) | (metadata[:, 1] >= self.heads) | (metadata[:, 0] < 0)
                | (metadata[:, 0] >= layers)).any():
            raise AssertionError("Recall changed logical time or inserted an incorrect slot count")
        flat = metadata[:, 0] * self.heads + metadata[:, 1]
        order = np.lexsort((metadata[:, 2], flat))
        flat_sorted = flat[order]
        heads, first, counts = np.unique(flat_sorted, return_index=True, return_counts=True)
        lens = self.head_lens.reshape(-1)
        need = int((lens[heads] + counts).max())
        if need > self.capacity:
            self._grow(max(need - self.capacity, 256, self.capacity // 8))
        rank = np.arange(len(order)) - np.repeat(first, counts)  # each entry's place within its head
        positions_sorted = metadata[order, 2]
        if ((flat_sorted[1:] == flat_sorted[:-1]) & (positions_sorted[1:] == positions_sorted[:-1])).any():
            raise ValueError("Cannot merge duplicate physical KV identities")
        rounds = int((counts.max() + self.INSERT_MAX - 1) // self.INSERT_MAX)
        rows_all = upload(order, self.device)
        recalled_all = payload.index_select(0, rows_all).contiguous()
        positions_all = upload(positions_sorted.astype(np.float32), self.device)
        batches = []
        for r in range(rounds):
            picked = np.flatnonzero((rank >= r * self.INSERT_MAX) & (rank < (r + 1) * self.INSERT_MAX))
            part_heads, part_first, part_counts = np.unique(flat_sorted[picked], return_index=True,
                                                            return_counts=True)
            plan = upload(np.stack([part_heads, part_first, part_counts], axis=1).astype(np.int64), self.device)
            if rounds > 1:
                index = upload(picked.astype(np.int64), self.device)
                recalled = recalled_all.index_select(0, index).contiguous()
                positions = positions_all.index_select(0, index).contiguous()
            else:
                recalled, positions = recalled_all, positions_all
            batches.append(((self.keys, self.values, self.positions, self.lengths, plan, recalled, positions),
                            part_heads, part_counts))
        # Every round is checked against the rows resident now before any
        # moves (the rounds' entries were checked against each other above).
        for args, _, _ in batches:
            state = int(operators().arena_insert(*args, True).item())
            if state & 1:
                raise ValueError("Cannot merge duplicate physical KV identities")
            if state:
                raise ValueError(f"arena recall refused (flag {state}): positions must ascend in every head")
        for args, part_heads, part_counts in batches:
            operators().arena_insert(*args, False)
            self._head_lens.reshape(-1)[part_heads] += part_counts
        return int(len(metadata))

    def check_flags(self) -> None:
        """Raise if a kernel flagged a full slot or a bad removal list (reads
        the device flags: a synchronisation)."""
        overflow, bad = self.flags.tolist()
        if overflow or bad:
            raise RuntimeError(f"arena kernels flagged: overflow={overflow}, bad removal list={bad}")
