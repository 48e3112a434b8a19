"""Low-level per-rank API: custom loss through autograd-attached logprobs,
optimizer steps, LoRA slots (snapshot, save, load, base)."""

import pytest
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


def test_extra_outputs_checkpoint_slots_and_planner(tmp_path):
    from art_mlx_b200.runtime.trainer_rank import plan_micro_batches

    torch.manual_seed(1)
    tr = GRPOTrainer(get_config("tiny-qwen3"), LoRASpec(r=8, alpha=16), "cpu", seed=0)
    rank = TrainerRank(tr)
    seq = torch.randint(0, 1024, (30,)).tolist()
    out = rank.forward([ForwardInput(tokens=seq, top_k=5, logits=True, hidden_states=True)])[0]
    # top-k: sorted, consistent with the full logits and with the target logprob
    logp = torch.log_softmax(out.logits.detach().float(), -1)
    ref_v, ref_i = logp.topk(5, dim=-1)
    assert torch.allclose(out.top_k.logprobs, ref_v, atol=1e-4) and torch.equal(out.top_k.tokens, ref_i)
    assert torch.allclose(logp.gather(1, out.targets[:, None])[:, 0], out.logprobs.detach(), atol=1e-4)
    assert out.hidden_states.shape == (29, tr.model.cfg.hidden_size) and out.hidden_states.requires_grad
    # two checkpoint slots trained in turn keep separate adapters and moments
    rank.save_checkpoint_slot("a")
    rank.save_checkpoint_slot("b")
    for name in ("a", "b", "a"):
        rank.set_checkpoint(name)
        rank.zero_grad()
        lp = rank.forward([ForwardInput(tokens=seq)])[0].logprobs
        (-(lp.mean() if name == "a" else -lp.mean())).backward()
        rank.optim_step(1e-2)
    rank.save_checkpoint_slot("a")
    sa, sb = rank.checkpoint_slot_optimizer_state("a"), rank.checkpoint_slot_optimizer_state("b")
    assert sa["step"] == 2 and sb["step"] == 1
    assert not torch.allclose(rank.checkpoints["a"]["master"], rank.checkpoints["b"]["master"])
    # a slot written to disk comes back with its optimizer state
    rank.set_checkpoint("b")
    rank.save_lora_slot(None, str(tmp_path / "b"))
    rank.load_checkpoint_slot("b2", str(tmp_path / "b"))
    assert torch.allclose(rank.checkpoints["b2"]["master"], rank.checkpoints["b"]["master"])
    assert rank.checkpoint_slot_optimizer_state("b2")["step"] == 1
    # planner: budget respected, order kept, oversize inputs alone
    assert plan_micro_batches([10, 10, 10, 50, 5], 25 * 4, 4) == [[0, 1], [2], [3], [4]]
    groups = list(rank.forward_micro_batches([ForwardInput(tokens=seq), ForwardInput(tokens=seq[:20])]))
    assert sum(len(g) for g, _ in groups) == 2


def test_prefix_tree_rows_refuse_positions_that_end_a_branch():
    """A scored position is valid only if the next row token continues it."""
    from art_mlx_b200.preprocessing.prefix_tree import prefix_tree_pack

    tr = GRPOTrainer(get_config("tiny-qwen3"), LoRASpec(r=4, alpha=8), "cpu", seed=0)
    rank = TrainerRank(tr)
    p = torch.tensor([1, 2, 3, 4])
    a, b = torch.cat([p, torch.tensor([10, 11])]), torch.cat([p, torch.tensor([20, 21, 22])])
    pk = prefix_tree_pack([a, b], max_depth=8, shareable_lengths=[3, 3])  # last prompt token in each branch
    row = dict(tokens=pk.tokens[0].tolist(), group_ids=pk.group_ids[0].tolist(),
               parent_ids=pk.parent_ids[0].tolist(), positions=pk.position_ids[0].tolist())
    ok = rank.forward([ForwardInput(score_positions=[3, 4, 6, 7, 8], **row)])[0]
    assert ok.targets.tolist() == [10, 11, 20, 21, 22]
    with pytest.raises(ValueError):
        rank.forward([ForwardInput(score_positions=[4, 5], **row)])  # 5 ends branch one; row token 6 is not its
