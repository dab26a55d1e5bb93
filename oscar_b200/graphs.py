"""CUDA-graph capture of one backend forward, for repeated steps of a fixed
batch geometry.

One OSCAR forward is about seven kernels (q/k/v rotation, INT2 store, staging
winner + write, tensor-core attention, split merge, output rotation) behind a
Python backend and a C ABI that plans the attention grid on the host.  At
decode sizes the device finishes a layer in tens of microseconds while the
host needs a few hundred to issue it; vLLM removes that cost by replaying
decode steps from CUDA graphs, and :class:`GraphedForward` does the same for
this backend.

Contract.  Capture takes static tensors: query / key / value / output and the
attention metadata (its device ``slot_mapping``, ``query_start_loc`` and
``seq_lens``).  Before each :meth:`GraphedForward.replay` the caller writes
the step's inputs into those tensors; the output tensor holds the result
afterwards.  The attention plan (requests, query lengths, sequence lengths,
history splits) is computed on the host at capture and is part of the graph:
replay only steps of the same batch geometry, and capture again when it
changes.  The staging window runs its graph-safe variant (seat scratch
cleared per call), so replays with new slot mappings stay correct.
"""
from __future__ import annotations

import torch


class GraphedForward:
    """``impl.forward(layer, query, key, value, kv_cache, attn_metadata,
    output=output)`` captured once, replayed per step.  ``pool`` (from
    ``torch.cuda.graph_pool_handle()``) lets graphs replayed one after another
    on one stream share their memory."""

    def __init__(self, impl, layer, query, key, value, kv_cache, attn_metadata, output, warmup: int = 2,
                 pool=None):
        if not torch.cuda.is_available() or query.device.type != "cuda":
            raise ValueError("GraphedForward needs CUDA tensors")
        self.args = (layer, query, key, value, kv_cache, attn_metadata)
        self.output = output
        self.impl = impl
        dev = query.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            # warm-up on a side stream: lazy set-up (staging arena, cached rotations,
            # kernel attributes) happens outside the capture
            for _ in range(max(1, warmup)):
                impl.forward(*self.args, output=output)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, pool=pool):
            impl.forward(*self.args, output=output)

    def replay(self) -> torch.Tensor:
        """Run the captured forward on the current contents of the static
        inputs; returns the static output tensor."""
        self.graph.replay()
        return self.output


class GraphedSequence:
    """Several backend forwards captured in order into one CUDA graph — the
    attention layers of a model step, as vLLM captures a whole model forward —
    so one launch replays all of them and consecutive layers' kernels overlap
    through programmatic dependent launch.  ``calls``: a list of
    ``(impl, layer, query, key, value, kv_cache, attn_metadata, output)``
    tuples under the same contract as :class:`GraphedForward` (static tensors,
    fixed batch geometry per call); a layer may appear more than once."""

    def __init__(self, calls, warmup: int = 1, pool=None):
        if not calls:
            raise ValueError("GraphedSequence needs at least one forward")
        if not torch.cuda.is_available() or calls[0][2].device.type != "cuda":
            raise ValueError("GraphedSequence needs CUDA tensors")
        self.calls = list(calls)
        dev = self.calls[0][2].device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            seen = set()
            for impl, layer, q, k, v, cache, md, out in self.calls:
                if id(layer) in seen:
                    continue
                seen.add(id(layer))
                for _ in range(max(1, warmup)):
                    impl.forward(layer, q, k, v, cache, md, output=out)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, pool=pool):
            for impl, layer, q, k, v, cache, md, out in self.calls:
                impl.forward(layer, q, k, v, cache, md, output=out)

    def replay(self) -> None:
        """Run every captured forward, in order, on the current contents of
        their static inputs."""
        self.graph.replay()
