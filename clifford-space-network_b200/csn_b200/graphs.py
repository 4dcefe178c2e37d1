"""A whole training step (forward, backward, optimizer step) as one CUDA graph.

The LM training step launches several hundred kernels (the fused block kernels of this
package, cuBLAS GEMMs, torch's elementwise and optimizer kernels).  Eagerly, each costs a
host launch, and the LMs' diagnostics read (one device -> host copy of the loss terms,
python/clifford_cl6.py:279-295 returns them as floats) stalls the host between forward and
backward.  ``TrainStepGraph`` captures the step once on static input buffers and replays it
with one launch; inside it the LMs return their diagnostics as device scalars
(``deferred_diagnostics``), read after the replay with one copy (``read``).

Requirements (checked): the model is on CUDA and the optimizer, if any, was built with
``capturable=True`` (its step count then lives on the device).  Without an optimizer the graph
is forward + backward, gradients left in ``.grad``.  The step's shapes are fixed at capture;
new inputs are copied into the static buffers.
"""
import contextlib
import threading
from typing import Callable, Dict, Optional, Sequence

import torch

_state = threading.local()


def diagnostics_deferred() -> bool:
    """True inside ``deferred_diagnostics()``: the LMs return diagnostics as device scalars."""
    return getattr(_state, "defer", False)


@contextlib.contextmanager
def deferred_diagnostics():
    prev = diagnostics_deferred()
    _state.defer = True
    try:
        yield
    finally:
        _state.defer = prev


def read(diagnostics: Dict[str, object]) -> Dict[str, float]:
    """{name: float} of a diagnostics dict of device scalars, with one device -> host copy."""
    keys = list(diagnostics)
    tens = [k for k in keys if torch.is_tensor(diagnostics[k])]
    out = {k: float(diagnostics[k]) for k in keys if k not in tens}
    if tens:
        vals = torch.stack([diagnostics[k].detach().float().reshape(()) for k in tens]).tolist()
        out.update(zip(tens, vals))
    return {k: out[k] for k in keys}


class TrainStepGraph:
    """zero_grad + ``loss_fn(model(*inputs))`` + backward + ``optimizer.step()`` as one graph.

    ``model(*inputs)`` must return ``(logits, loss, diagnostics)`` like the LMs of this
    package, or set ``loss_index`` / pass ``loss_fn`` for another output layout.  Call the
    object with inputs of the captured shapes: they are copied into the static buffers, the
    graph is replayed and the step's outputs (static tensors, overwritten by the next call)
    are returned.
    """

    def __init__(self, model: torch.nn.Module, optimizer: Optional[torch.optim.Optimizer],
                 example_inputs: Sequence[torch.Tensor], loss_fn: Optional[Callable] = None,
                 loss_index: int = 1, warmup: int = 3, inputs_require_grad: bool = False):
        if optimizer is not None:
            for group in optimizer.param_groups:
                if not group.get("capturable", False):
                    raise ValueError("TrainStepGraph: build the optimizer with capturable=True")
        dev = next(model.parameters()).device
        if dev.type != "cuda":
            raise ValueError("TrainStepGraph: the model must be on a CUDA device")
        self.model, self.optimizer = model, optimizer
        self.loss_fn, self.loss_index = loss_fn, loss_index
        self.inputs = [x.detach().to(dev).clone().requires_grad_(inputs_require_grad) for x in example_inputs]
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), deferred_diagnostics():
            for _ in range(max(1, warmup)):  # workspaces, cuBLAS handles, optimizer state
                self._zero_grad()
                self._body()
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        self._zero_grad()
        with torch.cuda.graph(self.graph), deferred_diagnostics():
            self.outputs = self._body()

    def _zero_grad(self):
        # gradients as None before capture: the captured backward writes them, it does not add
        if self.optimizer is not None:
            self.optimizer.zero_grad(set_to_none=True)
        self.model.zero_grad(set_to_none=True)
        for x in self.inputs:
            x.grad = None

    def _body(self):
        out = self.model(*self.inputs)
        loss = self.loss_fn(out) if self.loss_fn is not None else out[self.loss_index]
        loss.backward()
        if self.optimizer is not None:
            self.optimizer.step()
        return out

    def __call__(self, *inputs: torch.Tensor):
        if len(inputs) != len(self.inputs):
            raise ValueError(f"TrainStepGraph: expected {len(self.inputs)} inputs, got {len(inputs)}")
        for buf, x in zip(self.inputs, inputs):
            if x.shape != buf.shape:
                raise ValueError(f"TrainStepGraph: input shape {tuple(x.shape)} != captured {tuple(buf.shape)}")
            if x.data_ptr() != buf.data_ptr():
                with torch.no_grad():
                    buf.copy_(x, non_blocking=True)
        self.graph.replay()
        return self.outputs
