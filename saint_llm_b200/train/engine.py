"""Training-step engine for the CUDA path (used by ``bench.py`` and ``smoke()``).

Mixed precision layout: parameters in bf16 (the tensor-core operand type), one fp32
``main_grad`` buffer per parameter.  The native GEMM epilogues accumulate weight
gradients straight into ``main_grad``; gradients that autograd produces the normal
way (norm weights, embeddings, small gate parameters) are folded into ``main_grad``
by a post-accumulate hook and their bf16 ``.grad`` is dropped immediately.  The
optimizer (``MuonAdamW``) reads ``main_grad``.

The stacked expert weights get a joint ``(2, E, I, D)`` gate/up gradient buffer so
the grouped wgrad GEMM writes both halves in one launch.
"""

from __future__ import annotations

from collections.abc import Iterator

import torch
from torch import Tensor, nn


def cast_params(model: nn.Module, dtype: torch.dtype = torch.bfloat16) -> nn.Module:
    for p in model.parameters():
        if p.is_floating_point():
            p.data = p.data.to(dtype)
    return model


def _move_grad_hook(p: Tensor) -> None:
    if p.grad is not None:
        p.main_grad.add_(p.grad)  # type: ignore[attr-defined]
        p.grad = None


def attach_main_grads(model: nn.Module) -> list[Tensor]:
    """Create fp32 main_grad buffers and the hooks that fold autograd grads into them."""
    from saint_llm_b200.ops.moe import GroupedSwiGLUExperts

    for mod in model.modules():
        if isinstance(mod, GroupedSwiGLUExperts) and mod.gate_weight.requires_grad:
            joint = torch.zeros(2, *mod.gate_weight.shape, dtype=torch.float32, device=mod.gate_weight.device)
            mod.gate_weight.main_grad = joint[0]  # type: ignore[attr-defined]
            mod.up_weight.main_grad = joint[1]  # type: ignore[attr-defined]
    seen: set[int] = set()
    params: list[Tensor] = []
    for p in model.parameters():
        if not p.requires_grad or id(p) in seen:
            continue
        seen.add(id(p))
        if getattr(p, "main_grad", None) is None:
            p.main_grad = torch.zeros(p.shape, dtype=torch.float32, device=p.device)  # type: ignore[attr-defined]
        p.register_post_accumulate_grad_hook(_move_grad_hook)
        params.append(p)
    return params


def zero_main_grads(params: list[Tensor]) -> None:
    for p in params:
        p.main_grad.zero_()  # type: ignore[attr-defined]
        p.grad = None


def grad_of(p: Tensor) -> Tensor | None:
    mg = getattr(p, "main_grad", None)
    return mg if mg is not None else p.grad


class SyntheticTokens:
    """Uniform-random token batches generated on the host into pinned memory.

    ``n_batches`` distinct step batches (each ``(n_micro, micro_batch, seq_len)``) are
    drawn up front; ``batch(i)`` cycles through them, so consecutive steps train on
    different tokens (a single repeated batch would be memorised, and its loss would fall
    faster the fewer sequences a job trains on).  Every step's batch is copied
    host->device inside the timed region, like a data loader feeding the GPU.
    """

    def __init__(self, vocab: int, micro_batch: int, seq_len: int, n_micro: int, seed: int = 0,
                 n_batches: int = 1) -> None:
        g = torch.Generator().manual_seed(seed)
        bufs = torch.randint(0, vocab, (n_batches, n_micro, micro_batch, seq_len), generator=g, dtype=torch.int64)
        self.bufs = bufs.pin_memory() if torch.cuda.is_available() else bufs
        self.buf = self.bufs[0]
        self.n_micro = n_micro
        self.n_batches = n_batches

    def batch(self, i: int) -> Tensor:
        return self.bufs[i % self.n_batches]

    def __iter__(self) -> Iterator[Tensor]:
        yield from self.buf

    @property
    def bytes_per_step(self) -> int:
        return self.buf.numel() * self.buf.element_size()


__all__ = ["SyntheticTokens", "attach_main_grads", "cast_params", "grad_of", "zero_main_grads"]
