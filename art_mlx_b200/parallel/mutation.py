"""Deliberate faults for the sensitivity tests of the distributed oracle.

The distributed tests compare each parallel layout against one process.  Such
a comparison only proves something if it fails when a collective or a
normalisation goes wrong, so each switch below breaks one named step on
purpose and a test asserts that the comparison catches it (the role of the
mutation cases of the reference's oracle harness,
``tests/integration/megatron/model_support/oracle_harness.py:52-100``).

Switches are read from the environment variable ``ART_B200_MUTATION``
(comma-separated names) at each site, so spawned ranks inherit them; unset
(the default) means every path runs as written.  They change host-side
control only: no kernel is altered and no device fault is injected.
"""

from __future__ import annotations

import os

NAMES = {
    "dp_skip_grad_reduce": "the data-parallel gradient sum is skipped: each rank steps on its own gradient",
    "dp_local_token_normalization": "the loss is normalised by this rank's trainable tokens, not the step's",
    "tp_skip_reduce_scatter": "row-parallel partial sums are not reduced: each rank keeps its own partial",
    "ep_skip_combine_weights": "expert outputs are combined without the routing weights",
    "etp_skip_reduce_scatter": "the expert slices of the ETP group are not summed",
    "cp_skip_state_handoff": "gated DeltaNet pieces start from a zero state instead of their predecessor's",
}


def active(name: str) -> bool:
    assert name in NAMES, name
    raw = os.environ.get("ART_B200_MUTATION", "")
    return bool(raw) and name in raw.split(",")
