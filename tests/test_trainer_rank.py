"""Low-level per-rank API: custom loss through autograd-attached logprobs,
optimizer steps, LoRA slots (snapshot, save, load, base)."""

import torch

from art_mlx_b200.models.config import LoRASpec, get_config
from art_mlx_b200.runtime.trainer import GRPOTrainer
from art_mlx_b200.runtime.trainer_rank import ForwardInput, TrainerRank


def test_custom_objective_and_slots(tmp_path):
    torch.manual_seed(0)
    tr = GRPOTrainer(get_config("tiny-qwen3"), LoRASpec(r=8, alpha=16), "cpu", seed=0)
    rank = TrainerRank(tr)
    seqs = [torch.randint(0, 1024, (40,)).tolist(), torch.randint(0, 1024, (25,)).tolist()]
    inputs = [ForwardInput(tokens=seqs[0]), ForwardInput(tokens=seqs[1], score_positions=[10, 11, 12], entropy=True)]
    rank.snapshot_lora_slot("start")
    losses = []
    initial = None
    for _ in range(5):
        rank.zero_grad()
        outs = rank.forward(inputs)
        if initial is None:
            initial = outs[0].logprobs.detach().clone()
        assert outs[1].logprobs.shape == (3,) and outs[1].entropy is not None
        loss = -(outs[0].logprobs.mean() + outs[1].logprobs.mean())  # SFT-style objective
        loss.backward()
        assert float(tr.store.grad.abs().sum()) > 0
        rank.dp_reduce()
        rank.optim_step(3e-3)
        losses.append(float(loss))
    assert losses[-1] < losses[0]
    # the frozen slot reproduces the starting adapter, detached
    with rank.push_lora("start"):
        first = rank.forward(inputs[:1])[0].logprobs
    assert not first.requires_grad
    assert torch.allclose(first, initial, atol=1e-6)
    # save the live adapter, load it as a slot: identical logprobs
    rank.save_lora_slot(None, str(tmp_path / "live"))
    rank.load_lora_slot("live", str(tmp_path / "live"))
    live = rank.forward(inputs[:1])[0].logprobs.detach()
    with rank.push_lora("live"):
        again = rank.forward(inputs[:1])[0].logprobs
    assert torch.allclose(live, again, atol=1e-6)
    with rank.push_lora("base"):
        base = rank.forward(inputs[:1])[0].logprobs
    assert not torch.allclose(base, live, atol=1e-4)
