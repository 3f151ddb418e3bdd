"""CUDA-graph capture of a whole callable (the trunk), replayed with fresh inputs.

FoldForge's execution policy captures the trunk once and replays it
(``execution.cuda_graph`` with scope ``trunk``, ``src/foldforge/models/execution.py:196-260``).
The b200 kernels are capturable: they allocate nothing, never synchronise the host, and
take every buffer as an argument. Weights are packed on the eager warm-up call, before
capture.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence

import torch

Tensor = torch.Tensor


class GraphedCall:
    """``fn(*inputs)`` captured on static copies of ``example_inputs``.

    Calling the object copies the new inputs into the static buffers (same shapes and
    dtypes), replays the graph on the current stream and returns the static outputs
    (overwritten by the next call).
    """

    def __init__(self, fn: Callable[..., object], example_inputs: Sequence[Tensor], warmup: int = 1) -> None:
        self.fn = fn
        self.static_inputs = [t.clone() for t in example_inputs]
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream), torch.no_grad():
            for _ in range(warmup):
                fn(*self.static_inputs)
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.no_grad():
            self.static_outputs = fn(*self.static_inputs)
        torch.cuda.synchronize()

    def replay(self) -> object:
        """Replay on the inputs already in :attr:`static_inputs`."""
        self.graph.replay()
        return self.static_outputs

    def __call__(self, *inputs: Tensor) -> object:
        for dst, src in zip(self.static_inputs, inputs, strict=True):
            dst.copy_(src, non_blocking=True)
        return self.replay()
