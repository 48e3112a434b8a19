"""AdamW over the flat LoRA store (fused kernels on CUDA, same math on CPU).

Defaults are the reference trainer's (``src/art/dev/get_model_config.py:78-95``
and ``src/art/megatron/train.py:226-235``): betas (0.9, 0.99), weight decay
0.1, global grad-norm clip 0.1.  Clipping uses the norm of the full gradient
(over every rank's contribution once the gradient has been reduced).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..models.lora import LoRAStore
from ..ops import native


@dataclass
class AdamWConfig:
    beta1: float = 0.9
    beta2: float = 0.99
    eps: float = 1e-8
    weight_decay: float = 0.1
    max_grad_norm: float = 0.1


class FlatAdamW:
    def __init__(self, store: LoRAStore, cfg: AdamWConfig | None = None) -> None:
        self.store = store
        self.cfg = cfg or AdamWConfig()
        dev = store.device
        self._hp = torch.zeros(8, dtype=torch.float32, device=dev)
        self.grad_norm = torch.zeros(1, dtype=torch.float32, device=dev)

    def _hparams(self, lr: float, grad_scale: float, step: int) -> list[float]:
        c = self.cfg
        return [lr, c.beta1, c.beta2, c.eps, c.weight_decay, c.max_grad_norm, grad_scale, float(step)]

    def step(self, lr: float, grad_scale: float = 1.0, shard: tuple[int, int] | None = None) -> torch.Tensor:
        """One update; returns the (device) global grad norm after scaling.

        ``shard=(offset, numel)`` restricts the update to a slice of the flat
        buffers (the data-parallel partition); the norm is still global when
        the caller has reduced the full gradient.
        """
        st = self.store
        st.step += 1
        hp = self._hparams(lr, grad_scale, st.step)
        if st.device.type == "cuda":
            C = native.lib()
            self._hp.copy_(torch.tensor(hp, dtype=torch.float32), non_blocking=True)
            norm_sq = C.grad_sumsq(st.grad)
            sl = slice(None) if shard is None else slice(shard[0], shard[0] + shard[1])
            C.adamw_step(st.master[sl], st.compute[sl], st.grad[sl], st.exp_avg[sl],
                         st.exp_avg_sq[sl], self._hp, norm_sq, self.grad_norm)
            if shard is not None:
                st.grad.zero_()
        else:
            self._cpu_step(hp)
        st.version += 1
        return self.grad_norm

    def _cpu_step(self, hp: list[float]) -> None:
        lr, b1, b2, eps, wd, clip, gs, step = hp
        st = self.store
        g = st.grad * gs
        norm = torch.linalg.vector_norm(g)
        self.grad_norm.fill_(float(norm))
        if clip > 0 and norm > clip:
            g = g * (clip / (norm + 1e-6))
        st.exp_avg.mul_(b1).add_(g, alpha=1 - b1)
        st.exp_avg_sq.mul_(b2).addcmul_(g, g, value=1 - b2)
        bc1 = 1 - b1**step
        bc2 = 1 - b2**step
        st.master.mul_(1 - lr * wd)
        denom = (st.exp_avg_sq.sqrt() / (bc2**0.5)).add_(eps)
        st.master.addcdiv_(st.exp_avg, denom, value=-lr / bc1)
        if st.compute is not st.master:
            st.compute.copy_(st.master)
        st.grad.zero_()

    def state_dict(self) -> dict[str, torch.Tensor | int]:
        return {
            "exp_avg": self.store.exp_avg.detach().cpu(),
            "exp_avg_sq": self.store.exp_avg_sq.detach().cpu(),
            "step": self.store.step,
        }

    def load_state_dict(self, sd: dict) -> None:
        self.store.exp_avg.copy_(sd["exp_avg"])
        self.store.exp_avg_sq.copy_(sd["exp_avg_sq"])
        self.store.step = int(sd["step"])
