"""Forward traces with token UIDs.

A :class:`ForwardTraceCapture` passed in the forward context (``ctx["trace"]``)
records, for every decoder layer, the output of its token mixer (attention or
gated DeltaNet) and of its MLP / MoE block, plus the final hidden states, each
row tagged with the token's UID: its index in the full packed row.  Layouts
that split a row (context parallelism gives each rank a contiguous slice,
sequence parallelism a token shard) record only their rows, under their global
UIDs, so traces of any topology line up with a one-process oracle through
:func:`diff_traces`.

Reference: token-UID tracing (``ART_MEGATRON_ATTACH_TOKEN_UIDS``,
``src/art/megatron/training/trace.py:18-167``) and the forward-trace capture of
its topology oracle tests (``tests/integration/megatron/model_support/
forward_trace.py``).  ``ART_B200_TRACE_TOKEN_UIDS=1`` makes the trainer attach
UIDs to every micro step (``token_uids`` in the forward context).
"""

from __future__ import annotations

import os
from collections import defaultdict

import torch


def trace_token_uids_enabled() -> bool:
    return os.environ.get("ART_B200_TRACE_TOKEN_UIDS", "").strip().lower() in {"1", "true", "yes", "on"}


class ForwardTraceCapture:
    """Per-(layer, site) activations keyed by token UID, kept on the CPU in fp32."""

    def __init__(self, sites: tuple[str, ...] | None = None) -> None:
        self.sites = sites
        self.records: dict[tuple[int, str], list[tuple[torch.Tensor, torch.Tensor]]] = defaultdict(list)

    def record(self, layer: int, site: str, x: torch.Tensor, uids: torch.Tensor) -> None:
        if self.sites is not None and site not in self.sites:
            return
        self.records[(layer, site)].append((uids.detach().to("cpu", torch.int64),
                                            x.detach().to("cpu", torch.float32).reshape(x.shape[0], -1)))

    def gathered(self) -> dict[tuple[int, str], tuple[torch.Tensor, torch.Tensor]]:
        """``(uids, rows)`` per (layer, site), rows sorted by UID."""
        out = {}
        for key, parts in self.records.items():
            u = torch.cat([p[0] for p in parts])
            x = torch.cat([p[1] for p in parts])
            order = torch.argsort(u)
            out[key] = (u[order], x[order])
        return out

    def state(self) -> dict:
        """Plain tensors (for ``torch.save`` or an object all-gather)."""
        return {f"{k[0]}:{k[1]}": v for k, v in self.gathered().items()}

    @staticmethod
    def merge(states: list[dict]) -> dict:
        """Traces of several ranks (each its UID slice) as one trace."""
        acc: dict[str, list] = defaultdict(list)
        for st in states:
            for k, (u, x) in st.items():
                acc[k].append((u, x))
        out = {}
        for k, parts in acc.items():
            u = torch.cat([p[0] for p in parts])
            x = torch.cat([p[1] for p in parts])
            # a UID held by several ranks (tensor-parallel replicas) keeps its first copy
            first: dict[int, int] = {}
            for i, v in enumerate(u.tolist()):
                first.setdefault(int(v), i)
            keys = sorted(first)
            idx = torch.tensor([first[v] for v in keys], dtype=torch.long)
            out[k] = (torch.tensor(keys, dtype=torch.int64), x[idx])
        return out


def diff_traces(a: dict, b: dict) -> dict[str, float]:
    """Relative L2 difference per site over the UIDs both traces hold."""
    out = {}
    for k in sorted(set(a) & set(b), key=lambda s: (int(s.split(":")[0]), s)):
        ua, xa = a[k]
        ub, xb = b[k]
        common, ia, ib = _intersect(ua, ub)
        if common == 0:
            continue
        xa, xb = xa[ia], xb[ib]
        out[k] = float((xa - xb).norm() / (xb.norm() + 1e-12))
    return out


def _intersect(ua: torch.Tensor, ub: torch.Tensor):
    pos_b = {int(v): i for i, v in enumerate(ub.tolist())}
    ia, ib = [], []
    for i, v in enumerate(ua.tolist()):
        j = pos_b.get(int(v))
        if j is not None:
            ia.append(i)
            ib.append(j)
    return len(ia), torch.tensor(ia, dtype=torch.long), torch.tensor(ib, dtype=torch.long)
