"""CUDA-graph replay of the layer for a fixed token count (decode).

At decode sizes the layer's few kernels each take a few microseconds, so the
host's launch path (Python, ctypes, argument checks, one launch per kernel)
sets the pace.  ``GraphedMoE`` captures one ``kernel(...)`` call into a CUDA
graph with static input and output buffers and replays it: a replay costs one
graph launch.  The forward has no host synchronisation, so it captures as is: a
first call outside the capture sets the library up, and what the captured call
allocates (its output, and the workspace cached for the capture stream) comes
from the graph's private memory pool and stays with the graph.

    layer = GraphedMoE(weights, local_expert_offset=0, routed_scaling_factor=2.5, num_tokens=16)
    out = layer(routing_logits, routing_bias, hidden_states, hidden_states_scale)

``out`` is the graph's static output buffer: it is overwritten by the next call.
"""
from __future__ import annotations

import torch

from . import binding as B


class GraphedMoE:
    def __init__(self, weights, local_expert_offset: int, routed_scaling_factor: float, num_tokens: int,
                 device=None):
        w = weights
        self.device = torch.device(device) if device is not None else w.gemm1_weights.device
        self.offset = int(local_expert_offset)
        self.rsf = float(routed_scaling_factor)
        self.T = int(num_tokens)
        self.w = (w.gemm1_weights.contiguous(), w.gemm1_weights_scale.contiguous(), w.gemm2_weights.contiguous(),
                  w.gemm2_weights_scale.contiguous())
        d = self.device
        self.logits = torch.zeros((self.T, B.E_GLOBAL), dtype=torch.float32, device=d)
        self.bias = torch.zeros((B.E_GLOBAL,), dtype=torch.bfloat16, device=d)
        self.hidden = torch.zeros((self.T, B.H), dtype=torch.float8_e4m3fn, device=d)
        self.scale = torch.ones((B.H // 128, self.T), dtype=torch.float32, device=d)
        self.graph = None
        self.out = None

    def _run(self):
        return B.kernel(self.logits, self.bias, self.hidden, self.scale, *self.w, self.offset, self.rsf)

    def capture(self):
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._run()  # first call: the library's one-time device set-up (kernel attributes) runs outside the capture
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.out = self._run()
        self.graph = g
        return self

    def __call__(self, routing_logits, routing_bias, hidden_states, hidden_states_scale):
        if self.graph is None:
            self.capture()
        self.logits.copy_(routing_logits, non_blocking=True)
        self.bias.copy_(routing_bias.reshape(-1), non_blocking=True)
        self.hidden.copy_(hidden_states, non_blocking=True)
        self.scale.copy_(hidden_states_scale, non_blocking=True)
        self.graph.replay()
        return self.out
