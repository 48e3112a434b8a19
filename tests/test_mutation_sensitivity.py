"""Sensitivity of the distributed oracle: every parallel layout is compared
with one process in ``test_distributed.py``; here each comparison is rerun
with one collective or normalisation broken on purpose
(``art_mlx_b200.parallel.mutation``) and must fail.  CPU only (gloo ranks)."""

import os

import pytest
import torch

from art_mlx_b200.parallel.mutation import NAMES

from test_distributed import HYBRID_CPU, MOE_CPU, TP_CPU, _run, _single
from art_mlx_b200.models.config import get_config

CASES = [
    # (mutation, world, config name, config, tp, cp, etp)
    ("dp_skip_grad_reduce", 2, "tiny-qwen3", None, 1, 1, 1),
    ("dp_local_token_normalization", 2, "tiny-qwen3", None, 1, 1, 1),
    ("tp_skip_reduce_scatter", 2, "tp-tiny", TP_CPU, 2, 1, 1),
    ("ep_skip_combine_weights", 2, "moe-tiny", MOE_CPU, 1, 1, 1),
    ("etp_skip_reduce_scatter", 2, "moe-tiny", MOE_CPU, 1, 1, 2),
    ("cp_skip_state_handoff", 2, "hybrid-tiny", HYBRID_CPU, 1, 2, 1),
]


def test_every_mutation_has_a_case():
    assert {c[0] for c in CASES} == set(NAMES)


@pytest.mark.parametrize("name,world,cfg_name,cfg,tp,cp,etp", CASES, ids=[c[0] for c in CASES])
def test_oracle_catches_mutation(name, world, cfg_name, cfg, tp, cp, etp):
    os.environ["ART_B200_MUTATION"] = name
    try:
        res = _run(world, "gloo", cfg_name, tp_size=tp, cp_size=cp, etp_size=etp)
    finally:
        del os.environ["ART_B200_MUTATION"]
    master, metrics, _ = _single(torch.device("cpu"), cfg or get_config(cfg_name), "gloo")
    err = float((res["master"] - master).norm() / master.norm())
    dloss = abs(res["metrics"]["loss/train"] - metrics["loss/train"])
    # the unbroken comparison holds to 1e-5 on both (test_distributed.py)
    assert err > 1e-4 or dloss > 1e-4, (name, err, dloss)
