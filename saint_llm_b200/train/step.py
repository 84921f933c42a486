"""``TrainStep``: the public one-call training step of the CUDA engine.

``step = TrainStep(model, optimizer, micro_batches=32, params=...)``;
``loss = step(host_tokens)`` copies the step's token batch from (pinned) host memory
to the GPU, runs forward / backward over the micro-batches with fp32 gradient
accumulation, applies the optimizer and returns the mean loss as a Python float
(one device->host read).  ``step.run_device(device_tokens)`` is the same step without
the copies and the read (used for device-side timing).

``cuda_graph=True`` (single GPU, no gradient synchroniser): the forward + backward of one
micro-batch is captured once as a CUDA graph and replayed for every micro-batch, with the
micro-batch's tokens copied into the graph's static input first.  A micro-batch is a few
thousand kernel launches; replaying them as one graph removes the per-launch host cost
that otherwise leaves the GPU idle between small kernels.  The first call warms the step
up eagerly (two micro-batches whose gradients are discarded) and captures; the captured
micro-batch must not synchronise with the host (the CUDA path of the model does not).  If
the capture fails the step stays eager and ``graph_error`` says why.  The optimizer runs
eagerly after the replays.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
from torch import Tensor, nn

from saint_llm_b200.train.engine import zero_main_grads
from saint_llm_b200.train.losses import make_loss_fn
from saint_llm_b200.utils.profiling import phase


class TrainStep:
    def __init__(self, model: nn.Module, optimizer: torch.optim.Optimizer, *, micro_batches: int,
                 params: list[Tensor], loss_fn: nn.Module | None = None,
                 grad_sync: Callable[[list[Tensor]], None] | None = None, cuda_graph: bool = False) -> None:
        self.model = model
        self.optimizer = optimizer
        self.micro_batches = micro_batches
        self.params = params
        cfg = getattr(model, "cfg", None)
        self.loss_fn = loss_fn or make_loss_fn(cfg.mtp if cfg else None, moe_cfg=cfg.moe if cfg else None)
        self.grad_sync = grad_sync
        self.device = next(model.parameters()).device
        self.cuda_graph = cuda_graph and grad_sync is None and self.device.type == "cuda"
        self.graph_error: str | None = None
        self._graph: torch.cuda.CUDAGraph | None = None
        self._tok: Tensor | None = None
        self._total: Tensor | None = None

    # ------------------------------------------------------------------ eager
    def _micro_eager(self, tok: Tensor, last: bool, total: Tensor) -> None:
        with phase("forward"):
            loss = self.loss_fn(self.model, tok) / self.micro_batches
        hook = getattr(self.grad_sync, "before_last_backward", None)
        if hook is not None and last:
            hook()
        with phase("backward"):
            loss.backward()
        total += loss.detach()

    # ------------------------------------------------------------------ graphed
    def _capture(self, tok: Tensor) -> None:
        """Warm up on a side stream, then capture one micro-batch's forward + backward on it.

        The captured graph keeps its activations' memory for good (the optimizer can no
        longer reuse it between steps), so the capture is skipped when the warm-up's
        activation peak would not fit again next to what is allocated now plus a margin
        for the optimizer's temporaries."""
        self._tok = torch.zeros_like(tok)
        self._total = torch.zeros((), dtype=torch.float32, device=self.device)
        self._tok.copy_(tok)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        torch.cuda.synchronize(self.device)
        base = torch.cuda.memory_allocated(self.device)
        torch.cuda.reset_peak_memory_stats(self.device)
        with torch.cuda.stream(side):
            for _ in range(2):
                self._micro_eager(self._tok, False, self._total)
        torch.cuda.current_stream(self.device).wait_stream(side)
        zero_main_grads(self.params)  # the warm-up gradients are not part of any step
        torch.cuda.synchronize(self.device)
        act_peak = torch.cuda.max_memory_allocated(self.device) - base
        init_state = getattr(self.optimizer, "init_state", None)
        if init_state is not None:
            # the optimizer's buffers exist before the free memory is measured (created after
            # the warm-up, so they do not add to its peak)
            init_state()
        torch.cuda.empty_cache()
        free, _ = torch.cuda.mem_get_info(self.device)
        margin = 8 << 30
        if act_peak + margin > free:
            raise MemoryError(f"a captured micro-batch would pin {act_peak / 2**30:.1f} GiB of activations; "
                              f"{free / 2**30:.1f} GiB free")
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            loss = self.loss_fn(self.model, self._tok) / self.micro_batches
            loss.backward()
            self._total += loss.detach()
        del loss
        self._graph = graph

    def _micro_graphed(self, tokens: Tensor) -> Tensor:
        assert self._tok is not None and self._total is not None and self._graph is not None
        self._total.zero_()
        with phase("forward+backward (graph)"):
            for i in range(self.micro_batches):
                self._tok.copy_(tokens[i], non_blocking=True)
                self._graph.replay()
        return self._total.clone()

    # ------------------------------------------------------------------ public
    def run_device(self, tokens: Tensor) -> Tensor:
        """tokens: (micro_batches, mb, T) on the device.  Returns the mean loss (device scalar)."""
        self.model.train()
        if self.cuda_graph and self._graph is None and self.graph_error is None:
            try:
                self._capture(tokens[0])
            except Exception as e:  # noqa: BLE001 - any capture failure leaves the eager path
                self.graph_error = f"{type(e).__name__}: {e}".splitlines()[0][:300]
            if self._graph is None:  # failed or skipped: drop every trace of the attempt
                import gc

                self._tok = self._total = None
                zero_main_grads(self.params)
                gc.collect()
                torch.cuda.synchronize(self.device)
                torch.cuda.empty_cache()
        if self._graph is not None and self._tok is not None and tokens.shape[1:] == self._tok.shape:
            total = self._micro_graphed(tokens)
        else:
            total = torch.zeros((), dtype=torch.float32, device=self.device)
            for i in range(self.micro_batches):
                self._micro_eager(tokens[i], i == self.micro_batches - 1, total)
        if self.grad_sync is not None:
            with phase("grad_sync"):
                self.grad_sync(self.params)
        with phase("optimizer"):
            self.optimizer.step()
        post = getattr(self.grad_sync, "post_step", None)
        if post is not None:
            with phase("param_sync"):
                post()
        zero_main_grads(self.params)
        # the weights moved: re-quantise the cached FP8 copies now, outside any graph
        # capture, so replays (and the next eager forward) read current weights
        from saint_llm_b200.ops import fp8

        fp8.bump_weight_epoch()
        with phase("fp8_requant"):
            fp8.Fp8WeightCache.refresh_all()
        return total

    def __call__(self, host_tokens: Tensor) -> float:
        return float(self.run_device(host_tokens.to(self.device, non_blocking=True)).item())


__all__ = ["TrainStep"]
