"""Replay of a captured call, for callers bound by per-call host cost.

A Python-level call into the library costs about 11-12 us of host work
(argument checks, the output allocation, the ctypes call, the launch). Small
problems, such as the MAPPO communication module on a few hundred episodes
(about 6 us of device time), are bound by it when called one at a time, e.g.
once per environment step of a rollout. ``GraphedCall`` captures one call of
any of this package's operations (or a function of several) in a CUDA graph
and replays it: each call then costs one graph launch, plus one
device-to-device copy per tensor argument that is not the example call's
own tensor.

    from tarmac_b200 import ops
    from tarmac_b200.graphs import GraphedCall
    step = GraphedCall(ops.comm_forward, x, w_qkv, b_qkv, w_proj, b_proj, 2)
    y = step(x_next, w_qkv, b_qkv, w_proj, b_proj, 2)   # copies x_next only

Rules:

* The example call's tensors become the graph's input buffers: the graph
  reads whatever they hold when it is replayed. Passing the same tensor
  objects again costs nothing (in-place updates to them, e.g. new weights
  after a training step, are seen); passing other tensors of the same shapes
  and dtypes copies them into those buffers, overwriting the example
  tensors' contents. Non-tensor arguments must equal the example's (they are
  baked into the graph).
* The result is the graph's static output: the next replay overwrites it, so
  clone it to keep it.
* The example call runs a few times on a side stream before the capture, so
  that one-time set-up inside the library (kernel attribute changes) happens
  outside the graph.
"""

from __future__ import annotations

import torch


class GraphedCall:
    """One call of ``fn(*args)`` captured in a CUDA graph and replayed."""

    def __init__(self, fn, *example_args, warmup: int = 2):
        tensors = [a for a in example_args if torch.is_tensor(a)]
        if not tensors or not all(t.is_cuda for t in tensors):
            raise ValueError("GraphedCall needs CUDA tensor arguments")
        dev = tensors[0].device
        self._fn = fn
        self._static = list(example_args)
        self._consts = [None if torch.is_tensor(a) else a for a in example_args]
        cur = torch.cuda.current_stream(dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                fn(*self._static)
        cur.wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.output = fn(*self._static)

    def __call__(self, *args):
        if len(args) != len(self._static):
            raise ValueError("GraphedCall: argument count differs from the example call")
        for dst, src, const in zip(self._static, args, self._consts):
            if torch.is_tensor(dst):
                if src is dst:
                    continue
                if not torch.is_tensor(src) or src.shape != dst.shape or src.dtype != dst.dtype:
                    raise ValueError("GraphedCall: a tensor argument's shape or dtype "
                                     "differs from the example call")
                dst.copy_(src, non_blocking=True)
            elif src != const:
                raise ValueError("GraphedCall: a non-tensor argument differs from the "
                                 "example call")
        self.graph.replay()
        return self.output
