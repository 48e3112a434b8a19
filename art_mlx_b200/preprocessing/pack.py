"""Packing tokenized results into fixed-length training rows.

Format and normalisations follow the reference
``src/art/preprocessing/pack.py:26-625``:

* ``PackedTensors`` is a dict of ``[num_rows, seq_len]`` tensors: tokens,
  group_ids, parent_ids, input_pos, assistant_mask, logprobs, advantages,
  weights (+ optional MoE routing replay);
* results are appended to the current row while the prefix-tree-packed row
  still fits ``seq_len``; rows are shuffled;
* weights are zeroed off-mask and normalised to mean 1 over the mask;
  ``advantage_balance`` scales one sign down; advantages are then divided by
  ``mean(|A| * w)`` over the mask;
* on disk each tensor is its own raw file, memory-mapped back with
  ``torch.from_file(shared=True)``.
"""

from __future__ import annotations

import dataclasses
import math
import os
import random
from dataclasses import dataclass
from typing import Callable, Any, NamedTuple, TypedDict

import numpy as np
import torch
from typing_extensions import NotRequired

from .prefix_tree import estimate_prefix_tree_packed_tokens, prefix_tree_layout, prefix_tree_pack
from .tokenize import TokenizedResult


@dataclass
class PackedMoeRoutingReplay:
    """Replayed expert ids ``[rows, S, layers, topk]`` with a coverage mask."""

    expert_indices: torch.Tensor
    token_mask: torch.Tensor
    num_layers: int
    topk: int
    num_experts: int
    # shared-prefix tokens whose routes a later sibling also carried, and how
    # many of those disagreed (per-layer expert sets differ; the first kept)
    shared_route_tokens: int = 0
    route_conflict_tokens: int = 0


class PackedTensors(TypedDict):
    tokens: torch.Tensor
    group_ids: torch.Tensor
    parent_ids: torch.Tensor
    input_pos: torch.Tensor
    assistant_mask: torch.Tensor
    logprobs: torch.Tensor
    advantages: torch.Tensor
    weights: torch.Tensor
    pixel_values: list[torch.Tensor | None]
    image_grid_thw: list[torch.Tensor | None]
    moe_routing_replay: PackedMoeRoutingReplay | None
    # set when only some rows were filled: the step's scored-token count
    trainable_tokens: NotRequired[int]


class DiskPackedTensors(TypedDict):
    dir: str
    num_sequences: int
    sequence_length: int
    pixel_values: NotRequired[tuple[int, list[int]]]
    image_grid_thw: NotRequired[tuple[int, list[int]]]


DISK_DTYPES: dict[str, torch.dtype] = {
    "tokens": torch.long,
    "group_ids": torch.long,
    "parent_ids": torch.long,
    "input_pos": torch.long,
    "assistant_mask": torch.bool,
    "logprobs": torch.float32,
    "advantages": torch.float32,
    "weights": torch.float32,
}


class _Item(NamedTuple):
    token_ids: tuple[int, ...]  # a tuple: the planner compares sequences lexicographically
    input_pos: np.ndarray  # int64
    assistant_mask: np.ndarray  # int64
    logprobs: np.ndarray  # float64
    advantage: float
    weight: float
    prompt_id: int
    shareable: int
    routes: tuple[Any, ...] | None
    tokens: np.ndarray  # int64 copy of token_ids


def _ints(v: Any) -> tuple:
    return tuple(v.tolist()) if isinstance(v, np.ndarray) else tuple(v)


def _item(r: TokenizedResult, seq_len: int) -> _Item:
    """The packer's view of a result: numpy arrays converted once, so the
    row packer works on them without per-row list conversions."""
    toks = np.asarray(r.token_ids, dtype=np.int64)
    am = np.asarray(r.assistant_mask, dtype=np.int64)
    lp = np.asarray(r.logprobs, dtype=np.float64)
    n = min(len(am), len(lp))
    hit = np.flatnonzero((am[:n] != 0) | ~np.isnan(lp[:n]))
    first = int(hit[0]) if hit.size else len(toks)
    share = min(int(r.prompt_length), max(first - 1, 0))
    it = _Item(
        _ints(r.token_ids),
        np.asarray(r.input_pos, dtype=np.int64),
        am,
        lp,
        float(r.advantage),
        float(r.weight),
        int(r.prompt_id),
        share,
        tuple(r.moe_routed_experts) if r.moe_routed_experts is not None else None,
        toks,
    )
    return _truncate(it, seq_len)


def _truncate(it: _Item, seq_len: int) -> _Item:
    if len(it.token_ids) <= seq_len:
        return it
    return it._replace(
        token_ids=it.token_ids[:seq_len],
        input_pos=it.input_pos[:seq_len],
        assistant_mask=it.assistant_mask[:seq_len],
        logprobs=it.logprobs[:seq_len],
        shareable=min(it.shareable, seq_len),
        routes=it.routes[:seq_len] if it.routes is not None else None,
        tokens=it.tokens[:seq_len],
    )


def _row_len(row: list[_Item], seq_len: int) -> int:
    """Packed length of a candidate row, planned on the token tuples directly
    (same plan as ``estimate_prefix_tree_packed_tokens``, no tensor round trip)."""
    from .prefix_tree import _plan_segments

    segs = _plan_segments([i.token_ids for i in row], seq_len,
                          [max(0, min(i.shareable, len(i.token_ids))) for i in row])
    return sum(s.end - s.start for s in segs)


def _pack_row(row: list[_Item], seq_len: int, share: bool) -> dict[str, list]:
    if not row:
        out = {k: [] for k in ("tokens", "group_ids", "parent_ids", "input_pos", "assistant_mask", "logprobs", "advantages", "weights", "routes")}
        out["route_stats"] = (0, 0)
        return out
    toks, tree_gids, tree_pids, _, per_seq = prefix_tree_layout(
        [i.token_ids for i in row], seq_len if share else 0,
        [max(0, min(i.shareable, len(i.token_ids))) if share else 0 for i in row],
    )
    # every packed slot belongs to the first sequence that reaches it; later
    # sequences sharing the slot must agree on it (vectorised per sequence)
    n = len(toks)
    owned = np.zeros(n, dtype=bool)
    pos = np.zeros(n, dtype=np.int64)
    mask = np.zeros(n, dtype=np.int64)
    lps = np.full(n, np.nan, dtype=np.float64)
    adv = np.zeros(n, dtype=np.float64)
    w = np.zeros(n, dtype=np.float64)
    routes: list[Any] = [None] * n
    n_shared_routes = n_conflicts = 0
    for k, it in enumerate(row):
        dst = per_seq[k]
        m = len(dst)
        if (toks[dst] != it.tokens[:m]).any():
            raise RuntimeError("Prefix-tree pack token assignment mismatch")
        ip, am, lp = it.input_pos[:m], it.assistant_mask[:m], it.logprobs[:m]
        shared = owned[dst]
        if shared.any():
            if (pos[dst[shared]] != ip[shared]).any():
                raise RuntimeError("Prefix-tree pack cannot share mismatched input positions")
            if (am[shared] != 0).any() or (~np.isnan(lp[shared])).any():
                raise RuntimeError("Prefix-tree pack attempted to share a trainable token")
            if it.routes is not None:
                for src in np.nonzero(shared)[0].tolist():
                    have = routes[int(dst[src])]
                    if src < len(it.routes) and have is not None:
                        n_shared_routes += 1
                        n_conflicts += int(not _same_routes(have, it.routes[src]))
        fresh = ~shared
        d = dst[fresh]
        owned[d] = True
        pos[d] = ip[fresh]
        mask[d] = am[fresh]
        lps[d] = lp[fresh]
        adv[d] = it.advantage
        w[d] = it.weight
        if it.routes is not None:
            for src in np.nonzero(fresh)[0].tolist():
                if src < len(it.routes):
                    routes[int(dst[src])] = it.routes[src]
    return {
        "tokens": toks[:seq_len],
        "group_ids": tree_gids[:seq_len],
        "parent_ids": tree_pids[:seq_len],
        "input_pos": pos[:seq_len],
        "assistant_mask": mask[:seq_len],
        "logprobs": lps[:seq_len],
        "advantages": adv[:seq_len],
        "weights": w[:seq_len],
        "routes": routes[:seq_len],
        "route_stats": (n_shared_routes, n_conflicts),
    }


def _same_routes(a: Any, b: Any) -> bool:
    """Same expert set in every layer (top-k order does not matter)."""
    x, y = np.asarray(a), np.asarray(b)
    return x.shape == y.shape and bool((np.sort(x, axis=-1) == np.sort(y, axis=-1)).all())


def _step_normalisation(rows: list[list[_Item]], advantage_balance: float) -> tuple[float, float, int]:
    """(weight scale, advantage scale, scored tokens) of a step from its
    sequences: weights are divided by their mean over masked tokens, then
    advantages by the mean of |advantage| x weight; scored tokens exclude a
    masked token at a row's first position (it has no predecessor)."""
    n = w = a = 0.0
    items = []
    first_masked = 0
    for row in rows:
        for k, it in enumerate(row):
            c = float(it.assistant_mask.sum())
            if k == 0 and len(it.assistant_mask) and it.assistant_mask[0]:
                first_masked += 1
            items.append((c, it.weight, it.advantage))
            n += c
            w += c * it.weight
    if n == 0:
        return 1.0, 1.0, 0
    mean_w = w / n
    for c, wt, adv in items:
        if advantage_balance > 0.0 and adv <= 0:
            adv *= 1 - advantage_balance
        elif advantage_balance < 0.0 and adv >= 0:
            adv *= 1 + advantage_balance
        a += c * abs(adv) * (wt / mean_w)
    mean_a = a / n
    return 1.0 / mean_w, (1.0 / mean_a if mean_a > 0 else 1.0), int(n) - first_masked


def _padded(rows: list, seq_len: int, value: Any, dtype: torch.dtype) -> torch.Tensor:
    out = torch.full((len(rows), seq_len), value, dtype=dtype)
    for r, vals in enumerate(rows):
        if len(vals):
            out[r, : len(vals)] = torch.as_tensor(np.asarray(vals)).to(dtype)
    return out


def packed_tensors_from_tokenized_results(
    tokenized_results: list[TokenizedResult],
    seq_len: int,
    pad_token_id: int = -100,
    truncate_long_results: bool = True,
    advantage_balance: float = 0.0,
    verbosity: int = 1,
    pack_results: bool = True,
    include_moe_routing: bool = False,
    rng: random.Random | None = None,
    rows_needed: Callable[[int], set[int]] | None = None,
) -> PackedTensors:
    """Pack tokenized results into prefix-tree rows (reference
    ``src/art/preprocessing/pack.py``).

    ``rows_needed(n_rows)`` (optional) names the rows the caller will read
    (a data-parallel rank's own rows): the others keep their place but are
    left empty, and the weight / advantage normalisation and the step's
    trainable-token count (``trainable_tokens``) come from the per-sequence
    sums instead of the filled rows, so every rank sees the same values."""
    rows: list[list[_Item]] = [[]]
    # upper bound of the current row's packed length: an added sequence grows
    # the prefix tree by at most its own length, so the exact (re-planned)
    # length is only needed once the bound passes seq_len; same decisions as
    # planning every candidate row
    bound = 0
    for r in tokenized_results:
        if len(r.token_ids) > seq_len and not truncate_long_results:
            continue
        if include_moe_routing and r.moe_routed_experts is None:
            raise RuntimeError("MoE routing replay requested but a result has no routes")
        if sum(r.assistant_mask[r.prompt_length :]) == 0:
            continue
        it = _item(r, seq_len)
        if rows[-1]:
            grown = bound + len(it.token_ids)
            if pack_results and grown > seq_len:
                grown = _row_len([*rows[-1], it], seq_len)
            if not pack_results or grown > seq_len:
                rows.append([])
                grown = len(it.token_ids)
        else:
            grown = len(it.token_ids)
        rows[-1].append(it)
        bound = grown
    (rng or random).shuffle(rows)
    keep = rows_needed(len(rows)) if rows_needed is not None else None
    packed = [_pack_row(row if keep is None or r in keep else [], seq_len, pack_results)
              for r, row in enumerate(rows)]

    mask = _padded([p["assistant_mask"] for p in packed], seq_len, 0, torch.bool)
    weights = _padded([p["weights"] for p in packed], seq_len, 0.0, torch.float32)
    weights = torch.where(mask, weights, torch.zeros_like(weights))
    adv = _padded([p["advantages"] for p in packed], seq_len, 0.0, torch.float32)
    adv = torch.where(mask, adv, torch.zeros_like(adv))
    if advantage_balance > 0.0:
        adv = torch.where(adv > 0, adv, adv * (1 - advantage_balance))
    elif advantage_balance < 0.0:
        adv = torch.where(adv < 0, adv, adv * (1 + advantage_balance))
    trainable = None
    if keep is None:
        if mask.any():
            weights[mask] /= weights[mask].mean()
            adv[mask] /= (adv[mask].abs() * weights[mask]).mean()
    else:
        # the whole step's normalisation from per-sequence sums: every masked
        # token of a sequence carries its weight and advantage, and no masked
        # token is shared between sequences
        w_scale, a_scale, trainable = _step_normalisation(rows, advantage_balance)
        weights *= w_scale
        adv *= a_scale

    out: PackedTensors = {
        "tokens": _padded([p["tokens"] for p in packed], seq_len, pad_token_id, torch.long),
        "group_ids": _padded([p["group_ids"] for p in packed], seq_len, -1, torch.long),
        "parent_ids": _padded([p["parent_ids"] for p in packed], seq_len, -1, torch.long),
        "input_pos": _padded([p["input_pos"] for p in packed], seq_len, 0, torch.long),
        "assistant_mask": mask,
        "logprobs": _padded([p["logprobs"] for p in packed], seq_len, float("nan"), torch.float32),
        "advantages": adv,
        "weights": weights,
        "pixel_values": [None] * len(packed),
        "image_grid_thw": [None] * len(packed),
        "moe_routing_replay": None,
    }
    if trainable is not None:
        out["trainable_tokens"] = trainable
    if include_moe_routing:
        replay = tensorize_routes([p["routes"] for p in packed], seq_len)
        replay.shared_route_tokens = sum(p["route_stats"][0] for p in packed)
        replay.route_conflict_tokens = sum(p["route_stats"][1] for p in packed)
        out["moe_routing_replay"] = replay
    return out


def tensorize_routes(rows: list[list[Any]], seq_len: int) -> PackedMoeRoutingReplay:
    first = next((r for row in rows for r in row if r is not None), None)
    if first is None:
        raise RuntimeError("No MoE routes were packed")
    L, K = len(first), len(first[0])
    idx = torch.zeros(len(rows), seq_len, L, K, dtype=torch.int32)
    have = torch.zeros(len(rows), seq_len, dtype=torch.bool)
    for b, row in enumerate(rows):
        for s, route in enumerate(row[:seq_len]):
            if route is None:
                continue
            t = torch.as_tensor(route, dtype=torch.int32)
            if tuple(t.shape) != (L, K):
                raise RuntimeError("Packed MoE routes must have one rectangular shape")
            idx[b, s] = t
            have[b, s] = True
    return PackedMoeRoutingReplay(idx, have, L, K, max(K, int(idx.max().item()) + 1))


def select_rows(packed: PackedTensors, rows: list[int]) -> PackedTensors:
    """The packed rows ``rows`` as a new PackedTensors (one optimizer step's
    share when a train call is split into several gradient steps)."""
    idx = torch.tensor(rows, dtype=torch.long)
    out: dict[str, Any] = {}
    for key, val in packed.items():
        if isinstance(val, torch.Tensor):
            out[key] = val.index_select(0, idx)
        elif isinstance(val, list):
            out[key] = [val[r] for r in rows]
        elif isinstance(val, PackedMoeRoutingReplay):
            out[key] = dataclasses.replace(val, expert_indices=val.expert_indices.index_select(0, idx),
                                           token_mask=val.token_mask.index_select(0, idx))
        else:
            out[key] = val
    return out  # type: ignore[return-value]


def packed_tensors_from_dir(**kwargs: Any) -> PackedTensors:
    d = kwargs["dir"]
    n, s = kwargs["num_sequences"], kwargs["sequence_length"]
    os.makedirs(d, exist_ok=True)
    out: dict[str, Any] = {
        key: torch.from_file(f"{d}/{key}.pt", shared=True, size=n * s, dtype=dt).view(n, s)
        for key, dt in DISK_DTYPES.items()
    }
    out["pixel_values"] = [None] * n
    out["image_grid_thw"] = [None] * n
    out["moe_routing_replay"] = None
    rp = f"{d}/moe_routing_replay.pt"
    if os.path.exists(rp):
        out["moe_routing_replay"] = PackedMoeRoutingReplay(**torch.load(rp))
    return out  # type: ignore[return-value]


def packed_tensors_to_dir(tensors: PackedTensors, dir: str) -> DiskPackedTensors:
    disk: DiskPackedTensors = {
        "dir": dir,
        "num_sequences": int(tensors["tokens"].shape[0]),
        "sequence_length": int(tensors["tokens"].shape[1]),
    }
    mapped = packed_tensors_from_dir(**disk)
    for key in DISK_DTYPES:
        mapped[key].copy_(tensors[key])  # type: ignore[literal-required]
    rr = tensors.get("moe_routing_replay")  # type: ignore[attr-defined]
    rp = f"{dir}/moe_routing_replay.pt"
    if rr is not None:
        torch.save(dataclasses.asdict(rr), rp)
    elif os.path.exists(rp):
        os.remove(rp)
    return disk
