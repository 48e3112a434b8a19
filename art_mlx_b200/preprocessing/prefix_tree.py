"""Radix-tree (shared-prefix) packing of token sequences.

Same semantics as the reference ``src/art/megatron/prefix_tree_packing.py:27-112``:
sequences that start with the same tokens share that segment once; the walk
emits segments in depth-first pre-order, so every segment's descendants are
contiguous right after it.  Each emitted segment gets a fresh ``group_id``;
its ``parent_id`` is the segment it continues (roots point at themselves).

The kernel-facing mask used by the attention kernels is derived from this
layout in :func:`visibility_ends`: key ``j`` is visible to query ``i`` iff
``j <= i < kend[j]``, where ``kend[j]`` is the end of the subtree of ``j``'s
segment.  That one interval per key expresses "full attention to ancestors,
causal inside the own segment" with no per-pair metadata.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable, Sequence

import numpy as np
import torch


@dataclass(frozen=True)
class PrefixTreePack:
    tokens: torch.Tensor  # [1, L]
    group_ids: torch.Tensor  # [1, L]
    parent_ids: torch.Tensor  # [1, L]
    position_ids: torch.Tensor  # [1, L]
    positions_by_sequence: tuple[torch.Tensor, ...]


@dataclass(frozen=True)
class Segment:
    members: tuple[int, ...]
    start: int
    end: int
    group_id: int
    parent_id: int


def _plan_segments(
    rows: Sequence[Sequence[int]], max_depth: int, share_limits: Sequence[int]
) -> list[Segment]:
    lengths = [len(r) for r in rows]
    out: list[Segment] = []
    next_id = [1]

    def emit(members: tuple[int, ...], start: int, end: int, parent: int | None) -> int:
        gid = next_id[0]
        next_id[0] += 1
        out.append(Segment(members, start, end, gid, gid if parent is None else parent))
        return gid

    def common_end(members: tuple[int, ...], start: int) -> int:
        limit = min(min(lengths[m], share_limits[m]) for m in members)
        # the lexicographic min and max of a set agree on a position iff all do
        lo = min((rows[m] for m in members))
        hi = max((rows[m] for m in members))
        pos = start
        while pos < limit and lo[pos] == hi[pos]:
            pos += 1
        return pos

    def split_by_next_token(members: tuple[int, ...], start: int) -> list[tuple[int, ...]]:
        buckets: dict[int, list[int]] = {}
        for m in members:
            buckets.setdefault(rows[m][start], []).append(m)
        return [tuple(v) for v in buckets.values()]  # insertion (first-seen) order

    # explicit stack instead of recursion: deep trees must not hit the
    # interpreter recursion limit.  Frames are processed in pre-order.
    stack: list[tuple[tuple[int, ...], int, int | None, int]] = [
        (tuple(range(len(rows))), 0, None, 0)
    ]
    while stack:
        members, start, parent, depth = stack.pop()
        active = tuple(m for m in members if lengths[m] > start)
        if not active:
            continue
        shareable = tuple(m for m in active if share_limits[m] > start)
        for m in active:
            if m not in shareable:
                emit((m,), start, lengths[m], parent)
        if not shareable:
            continue
        if max_depth == 0 or len(shareable) == 1 or (
            parent is not None and depth >= max_depth
        ):
            for m in shareable:
                emit((m,), start, lengths[m], parent)
            continue
        end = common_end(shareable, start)
        if end > start:
            gid = emit(shareable, start, end, parent)
            stack.append((shareable, end, gid, depth + 1))
            continue
        for sub in reversed(split_by_next_token(shareable, start)):
            stack.append((sub, start, parent, depth))
    return out


def _as_row(t: torch.Tensor) -> torch.Tensor:
    if t.ndim != 1:
        raise ValueError(f"prefix_tree_pack expects 1-D tensors, got {tuple(t.shape)}")
    return t.detach().to(dtype=torch.long).contiguous()


def _limits(tensors: Sequence[torch.Tensor], limits: Iterable[int] | None) -> list[int]:
    if limits is None:
        return [int(t.numel()) for t in tensors]
    vals = [int(v) for v in limits]
    if len(vals) != len(tensors):
        raise ValueError(
            "shareable_lengths must have one entry per sequence, "
            f"got {len(vals)} for {len(tensors)} sequences"
        )
    return [max(0, min(v, int(t.numel()))) for v, t in zip(vals, tensors)]


def prefix_tree_layout(
    rows: Sequence[Sequence[int]], max_depth: int, share_limits: Sequence[int]
) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray, list[np.ndarray]]:
    """Packed layout of token sequences (lists or tuples) as numpy arrays:
    ``(tokens, group_ids, parent_ids, position_ids, positions_by_sequence)``."""
    segs = _plan_segments(rows, max_depth, share_limits)
    n_total = sum(s.end - s.start for s in segs)
    toks = np.empty(n_total, np.int64)
    gids = np.empty(n_total, np.int64)
    pids = np.empty(n_total, np.int64)
    pos = np.empty(n_total, np.int64)
    per_seq: list[list[np.ndarray]] = [[] for _ in rows]
    base = 0
    for s in segs:
        n = s.end - s.start
        toks[base : base + n] = rows[s.members[0]][s.start : s.end]
        gids[base : base + n] = s.group_id
        pids[base : base + n] = s.parent_id
        pos[base : base + n] = np.arange(s.start, s.end)
        span = np.arange(base, base + n, dtype=np.int64)
        for m in s.members:
            per_seq[m].append(span)
        base += n
    seqs = [np.concatenate(p) if p else np.zeros(0, np.int64) for p in per_seq]
    return toks, gids, pids, pos, seqs


def prefix_tree_pack(
    sequences: Iterable[torch.Tensor],
    *,
    max_depth: int,
    shareable_lengths: Iterable[int] | None = None,
) -> PrefixTreePack:
    """Pack 1-D token tensors into one row, storing shared prefixes once.

    ``max_depth=0`` disables sharing; ``shareable_lengths`` caps how much of
    each sequence may be shared (trainable tokens are never shared).
    """
    if max_depth < 0:
        raise ValueError("max_depth must be >= 0")
    tensors = [_as_row(s) for s in sequences]
    if not tensors:
        e = torch.empty(1, 0, dtype=torch.long)
        return PrefixTreePack(e, e, e, e, ())
    rows = [t.tolist() for t in tensors]
    toks, gids, pids, pos, per_seq = prefix_tree_layout(rows, max_depth, _limits(tensors, shareable_lengths))
    as_row = lambda v: torch.from_numpy(v).unsqueeze(0)  # noqa: E731
    return PrefixTreePack(
        tokens=as_row(toks),
        group_ids=as_row(gids),
        parent_ids=as_row(pids),
        position_ids=as_row(pos),
        positions_by_sequence=tuple(torch.from_numpy(p) for p in per_seq),
    )


def estimate_prefix_tree_packed_tokens(
    sequences: Iterable[torch.Tensor],
    *,
    max_depth: int,
    shareable_lengths: Iterable[int] | None = None,
) -> int | None:
    """Exact packed length without building tensors (CPU tensors only)."""
    if max_depth < 0:
        raise ValueError("max_depth must be >= 0")
    tensors = []
    for s in sequences:
        t = _as_row(s)
        if t.device.type != "cpu":
            return None
        tensors.append(t)
    rows = [t.tolist() for t in tensors]
    segs = _plan_segments(rows, max_depth, _limits(tensors, shareable_lengths))
    return sum(s.end - s.start for s in segs)


# ---------------------------------------------------------------------------
# Parsing packed rows back into segments, and the kernel-facing mask.
# ---------------------------------------------------------------------------


@dataclass(frozen=True)
class TreeSegment:
    group_id: int
    parent_id: int
    start: int
    end: int
    ancestors: tuple[int, ...]
    subtree_end: int


def parse_prefix_tree_row(group_ids: torch.Tensor, parent_ids: torch.Tensor) -> list[TreeSegment]:
    """Split one packed row into contiguous group runs and resolve ancestry.

    Padding (``group_id == -1``) ends the valid region.  Raises if a group id
    repeats non-contiguously or a child precedes / overlaps its parent
    (the checks of the reference ``src/art/megatron/prefix_tree.py:29-140``).
    """
    g = group_ids.tolist()
    p = parent_ids.tolist()
    n = len(g)
    valid = n
    for i, v in enumerate(g):
        if v == -1:
            valid = i
            break
    runs: list[tuple[int, int, int, int]] = []
    i = 0
    while i < valid:
        j = i
        while j < valid and g[j] == g[i] and p[j] == p[i]:
            j += 1
        runs.append((i, j, g[i], p[i]))
        i = j
    seen: dict[int, int] = {}
    segs: list[TreeSegment] = []
    for idx, (s, e, gid, pid) in enumerate(runs):
        if gid in seen:
            raise RuntimeError(f"prefix-tree group {gid} is not contiguous")
        seen[gid] = idx
        if gid == pid:
            anc: tuple[int, ...] = ()
        else:
            if pid not in seen:
                raise RuntimeError(f"group {gid} points to missing parent {pid}")
            parent = segs[seen[pid]]
            if parent.end > s:
                raise RuntimeError(f"parent {pid} must end before child {gid} starts")
            anc = (*parent.ancestors, pid)
        segs.append(TreeSegment(gid, pid, s, e, anc, e))
    # subtree ends: a segment's subtree runs until the next segment that is
    # not one of its descendants (pre-order layout).
    out: list[TreeSegment] = []
    for k, seg in enumerate(segs):
        end = seg.end
        for later in segs[k + 1 :]:
            if seg.group_id in later.ancestors:
                end = later.end
            else:
                break
        out.append(TreeSegment(seg.group_id, seg.parent_id, seg.start, seg.end, seg.ancestors, end))
    return out


def visibility_ends(group_ids: torch.Tensor, parent_ids: torch.Tensor) -> torch.Tensor:
    """Per-key visibility end ``kend`` for packed rows ``[B, S]`` (int32).

    Query ``i`` may attend key ``j`` iff ``j <= i < kend[j]``.  Padding keys
    get ``kend = j + 1`` (visible to themselves only, so padded query rows stay
    finite).  Works for any depth because the packer emits pre-order.
    """
    B, S = group_ids.shape
    out = torch.empty(B, S, dtype=torch.int32)
    for b in range(B):
        segs = parse_prefix_tree_row(group_ids[b], parent_ids[b])
        row = torch.arange(1, S + 1, dtype=torch.int32)
        for seg in segs:
            row[seg.start : seg.end] = seg.subtree_end
        out[b] = row
    return out


def dense_prefix_tree_mask(kend: torch.Tensor) -> torch.Tensor:
    """Boolean ``[B, S, S]`` mask (query, key) from visibility ends; test oracle."""
    S = kend.shape[-1]
    i = torch.arange(S).view(1, S, 1)
    j = torch.arange(S).view(1, 1, S)
    return (j <= i) & (i < kend.to(torch.long).unsqueeze(1))
