"""Device-side failure detection: bounded waits that run out are surfaced.

Every spin-wait of the framework's kernels (the cross-GPU peer barrier, the
tensor-core pipeline barriers) has a time and iteration limit; when it runs
out the kernel records a status word and returns instead of hanging.  The
trainer folds those words into the step's single metric read
(``StepMetrics.to_host``) and raises, so no checkpoint is published from a
step whose exchange was incomplete (reference counterpart: the worker's
failure detection, ``src/art/megatron/service.py`` heartbeat/exit checks;
the device side has no counterpart there because its waits live in NCCL).

The GPU test makes a wait run out without faulting anything: a one-GPU
peer barrier whose "peer" flag slot is an ordinary local buffer that nothing
ever writes, with a 2 ms limit.
"""

import time

import pytest
import torch

from art_mlx_b200.runtime.trainer import DeviceWaitTimeout, StepMetrics


def _metrics(health):
    z = torch.zeros(())
    return StepMetrics(loss=z, entropy=z, probs_corr=z, kl=z, grad_norm=z, n_train=4, n_tokens=8,
                       health=health, health_names=("dp_barrier", "tensor_core_wait"))


def test_to_host_passes_clean_status():
    m = _metrics(torch.zeros(2, dtype=torch.int32)).to_host()
    assert m["data/step_packed_tokens"] == 8.0 and m["data/step_trainer_tokens"] == 4.0


def test_to_host_raises_on_timed_out_wait():
    with pytest.raises(DeviceWaitTimeout, match="tensor_core_wait=3"):
        _metrics(torch.tensor([0, 3], dtype=torch.int32)).to_host()


@pytest.mark.gpu
def test_peer_barrier_timeout_is_recorded_and_raised(cuda):
    from art_mlx_b200.ops import native

    C = native.lib()
    mine = torch.zeros(64, dtype=torch.int32, device=cuda)  # this rank's flag slots
    fake_peer = torch.zeros(64, dtype=torch.int32, device=cuda)  # never signalled back
    flags = torch.tensor([mine.data_ptr(), fake_peer.data_ptr()], dtype=torch.int64, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    torch.cuda.synchronize()
    t0 = time.monotonic()
    C.peer_barrier(flags, 0, 2, 1, 2_000_000, status)  # rank 0 of 2, epoch 1, 2 ms limit
    torch.cuda.synchronize()
    elapsed = time.monotonic() - t0
    assert int(status.item()) == 1, "the wait on the silent peer must record a timeout"
    assert elapsed < 5.0
    assert int(mine[0].item()) == 1 and int(fake_peer[0].item()) == 1  # own arrivals were published
    # the context is still usable
    assert float((torch.ones(4, device=cuda) * 2).sum().item()) == 8.0
    # the trainer's metric read refuses the step
    z = torch.zeros((), device=cuda)
    m = StepMetrics(loss=z, entropy=z, probs_corr=z, kl=z, grad_norm=z, n_train=1, n_tokens=1,
                    health=status.clone(), health_names=("dp_barrier",))
    with pytest.raises(DeviceWaitTimeout, match="dp_barrier=1"):
        m.to_host()
    # a barrier whose peer did arrive completes with a clean status
    status.zero_()
    mine.zero_()
    fake_peer.zero_()
    mine[1] = 2  # the peer's arrival for epoch 2 is already there
    C.peer_barrier(flags, 0, 2, 2, 2_000_000, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0


@pytest.mark.gpu
def test_trainer_health_words_include_tensor_core_word(cuda):
    from art_mlx_b200.models.config import LoRASpec, get_config
    from art_mlx_b200.runtime.trainer import GRPOTrainer

    tr = GRPOTrainer(get_config("tiny-qwen3"), LoRASpec(r=4, alpha=8), cuda)
    names, words = tr.health_words()
    assert "tensor_core_wait" in names
    tr.check_health()  # clean
