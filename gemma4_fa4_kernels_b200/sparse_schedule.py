"""Exact block-sparse tile schedules of local (sliding-window) layers.

Restates the interface of the reference's ``sparse_schedule.py`` (the
``SparseTileRows`` / ``Gemma4LocalSparseSchedule`` containers and
``build_gemma4_local_sparse_schedule``, ``src/gemma4_fa4/sparse_schedule.py:
18-92, 291-374``) over the library's device planner (``g4_tile_schedule``):
the lists returned here are the ones the attention kernels iterate, so every
tile outside them is never loaded.  Differences from the reference, both from
the B200 kernel design:

* tiles are 128 x 128 in both directions (the reference's H100 kernels use
  128 x 80 forward and 64 x 64 backward tiles);
* every forward row also says which of its tiles are full (all pairs
  allowed), the tiles on which the kernels skip the mask, and which are text
  tiles (no vision key, one document for the tile's rows and keys), on which
  the window / causal range rule alone is exact and the kernels read no
  metadata.  The backward rows are the transpose (per key tile, the query
  tiles that reach it), which is how the key-major kernels walk the same
  incidence.
"""

from __future__ import annotations

import ctypes
from collections.abc import Sequence
from dataclasses import dataclass

import torch

from . import _lib
from .ops import _raise_for, _stream

TILE = 128
# key-tile list entries (include/gemma4_b200.h, g4_tile_schedule): the tile
# index in the low 30 bits, then the text and full tags
_ENTRY_INDEX = 0x3FFFFFFF
_ENTRY_TEXT = 0x40000000
_ENTRY_FULL = -0x80000000  # bit 31 of an int32 entry


@dataclass(frozen=True)
class SparseTileRows:
    """Ordered adjacency from row tiles to the column tiles that hold at least
    one allowed pair; ``full`` marks columns whose every pair is allowed,
    ``text`` those on which the window / causal range rule is exact."""

    rows: tuple[tuple[int, ...], ...]
    row_block_size: int
    column_block_size: int
    column_blocks: int
    full: tuple[tuple[bool, ...], ...] = ()
    text: tuple[tuple[bool, ...], ...] = ()

    def __post_init__(self) -> None:
        for row in self.rows:
            if tuple(sorted(set(row))) != row:
                raise ValueError("sparse row indices must be sorted and unique")
            if any(i < 0 or i >= self.column_blocks for i in row):
                raise ValueError("sparse row index is out of range")

    @property
    def candidate_pairs(self) -> int:
        return sum(len(r) for r in self.rows)

    @property
    def compact_width(self) -> int:
        return max([1] + [len(r) for r in self.rows])

    @property
    def storage_bytes(self) -> int:
        """INT32 compact storage: a count and the padded column list per row."""
        return 4 * len(self.rows) * (1 + self.compact_width)


@dataclass(frozen=True)
class Gemma4LocalSparseSchedule:
    """Forward (query tile -> key tiles) and transposed backward (key tile ->
    query tiles) schedules of one sequence."""

    q_length: int
    k_length: int
    forward: SparseTileRows
    backward: SparseTileRows

    @property
    def candidate_pairs(self) -> int:
        return self.forward.candidate_pairs

    def scheduled_score_slots(self, num_q_heads: int) -> int:
        """Score elements the kernels compute per pass (every listed tile is
        computed once per query head)."""
        if num_q_heads <= 0:
            raise ValueError("num_q_heads must be positive")
        return num_q_heads * self.forward.candidate_pairs * TILE * TILE


def _meta_tensor(values, k_length, name, device):
    if values is None:
        return None
    t = torch.as_tensor(values, dtype=torch.int32)
    if t.ndim != 1 or t.numel() != k_length:
        raise ValueError(f"{name} must have Sk = {k_length} entries")
    return t.to(device).contiguous()


def build_gemma4_local_sparse_schedule(
    vision_block_ids: Sequence[int] | torch.Tensor | None,
    document_ids: Sequence[int] | torch.Tensor | None,
    *,
    q_length: int,
    k_length: int,
    sliding_window: int = 1024,
    device: torch.device | str | None = None,
) -> Gemma4LocalSparseSchedule:
    """Exact schedule of one sequence (lower-right aligned queries), built by
    the device planner the attention kernels use.  ``vision_block_ids`` and
    ``document_ids`` follow the key stream (``Sk`` entries; ``None`` = text /
    one document)."""
    if q_length <= 0 or k_length <= 0 or q_length > k_length:
        raise ValueError("sparse scheduling requires 1 <= Sq <= Sk")
    if sliding_window <= 0:
        raise ValueError("sliding_window must be positive")
    device = torch.device(device if device is not None else "cuda")
    vis = _meta_tensor(vision_block_ids, k_length, "vision_block_ids", device)
    doc = _meta_tensor(document_ids, k_length, "document_ids", device)
    lib = _lib.load()
    a = _lib.G4AttnArgs()
    a.batch, a.seqlen_q, a.seqlen_k = 1, q_length, k_length
    a.num_q_heads = a.num_kv_heads = 1
    a.head_dim_qk = a.head_dim_v = 256
    a.window = int(sliding_window)
    a.vision_ids = None if vis is None else vis.data_ptr()
    a.document_ids = None if doc is None else doc.data_ptr()
    ws = torch.empty(max(256, lib.g4_tile_schedule_workspace_bytes(ctypes.byref(a))),
                     dtype=torch.uint8, device=device)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    nq, nk = -(-q_length // TILE), -(-k_length // TILE)
    counts = torch.empty(nq, dtype=torch.int32, device=device)
    keys = torch.empty(nq, nk, dtype=torch.int32, device=device)
    _raise_for(lib.g4_tile_schedule(ctypes.byref(a), counts.data_ptr(), keys.data_ptr(), nk,
                                    _stream(device)), "g4_tile_schedule")
    counts_h, keys_h = counts.cpu().tolist(), keys.cpu().tolist()
    rows, full, text = [], [], []
    for g in range(nq):
        ent = keys_h[g][:counts_h[g]]
        rows.append(tuple(e & _ENTRY_INDEX for e in ent))
        full.append(tuple(bool(e & _ENTRY_FULL) for e in ent))
        text.append(tuple(bool(e & _ENTRY_TEXT) for e in ent))
    cols = [[] for _ in range(nk)]
    for g, row in enumerate(rows):
        for kt in row:
            cols[kt].append(g)
    forward = SparseTileRows(tuple(rows), TILE, TILE, nk, tuple(full), tuple(text))
    backward = SparseTileRows(tuple(tuple(c) for c in cols), TILE, TILE, max(nq, 1))
    return Gemma4LocalSparseSchedule(q_length, k_length, forward, backward)
