"""Two-stream layer pipeline for one decode step.

A decode step runs, per layer, a short producer (the residency lookup, or the
lookup + victim selection + promotion of a host-backed request) followed by
the HBM-bound gather that reads the producer's output.  Layer i+1's producer
does not depend on layer i's gather, so the two can run at the same time when
the producer's blocks fit on the SMs beside the gather's (register and shared
memory budgets are sized for that: the gather leaves room for one producer
block per SM).

``LayerPipeline`` runs the producers in layer order on the caller's stream and
the consumers in layer order on a second stream, with one event per layer
between them; the caller's stream waits for the last consumer before the call
returns.  Consumers stay ordered among themselves, so the layers may share one
output buffer.  It works eagerly and under CUDA graph capture (the second
stream forks from and joins the caller's stream).

With ``wait=False`` a consumer does not wait for its producer.  That is for a
consumer that reads none of its producer's output -- the mapped gather resolves
each token's hot slot from the residency map itself, so layer i's lookup (whose
slots and miss list feed the swap-in) and layer i's gather can run at the same
time.  Then the consumers run back to back on the caller's stream (where
programmatic dependent launch chains them) and each producer is forked onto the
second stream at the start of its layer (it sees everything issued before
layer i, e.g. the work that produced layer i's Top-K, but not consumer i); the
caller's stream joins the second stream once, at the end.  It stays valid when
layer i's Top-K is only known once layer i-1 is done.
"""

from __future__ import annotations

from typing import Callable, Sequence

import torch

Launch = Callable[[int], None]


class LayerPipeline:
    """``produce[i](stream)`` then ``consume[i](stream)`` for every layer, with
    consumer i overlapping producer i+1, or with ``wait=False`` producer i alone
    (see module docstring)."""

    def __init__(self, produce: Sequence[Launch], consume: Sequence[Launch], device, *, wait: bool = True):
        self.produce, self.consume = list(produce), list(consume)
        if not self.produce or len(self.produce) != len(self.consume):
            raise ValueError("need one producer and one consumer per layer, at least one layer")
        self.device = torch.device(device)
        self.wait = bool(wait)
        self.side = torch.cuda.Stream(self.device)
        self.ready = [torch.cuda.Event() for _ in self.produce]

    def __call__(self) -> None:
        main = torch.cuda.current_stream(self.device)
        side = self.side
        side.wait_stream(main)  # fork: the second stream sees everything issued before the step
        main_handle, side_handle = main.cuda_stream, side.cuda_stream
        if self.wait:
            for produce, consume, ready in zip(self.produce, self.consume, self.ready):
                produce(main_handle)
                ready.record(main)
                side.wait_event(ready)
                consume(side_handle)
        else:
            for produce, consume, ready in zip(self.produce, self.consume, self.ready):
                ready.record(main)  # fork producer i off everything before layer i
                side.wait_event(ready)
                produce(side_handle)
                consume(main_handle)
        main.wait_stream(side)  # join
