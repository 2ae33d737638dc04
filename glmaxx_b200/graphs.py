"""Per-row-bucket CUDA graphs of one rank's routed-MoE step.

The reference engine replays one CUDA graph per row bucket of a step
(crates/glm-engine/src/graph.rs:13-80, GraphKey.verifier_row_bucket), with the
decode buckets 1..128 and the prefill buckets 256..3072 of
crates/glm-cli/src/profile.rs:10-11.  BucketedMoE captures the layer once per
bucket over fixed, bucket-sized prefixes of persistent input and output buffers;
a call with T rows copies them into the input buffer, zeroes the rows up to the
bucket and replays that bucket's graph.

Every stage of the step is independent per row (router, compaction order of
the real rows, per-row NVFP4 quantisation, per-element dot products, per-token
combine), and the decode path's shared-expert split-K layout depends only on
ceil(T / 64), which is the same for T and its bucket.  So on the deterministic
decode path (buckets <= 256) the real rows are the same bits as an unpadded
launch; the prefill path's atomic FC2 combine sums in a run-dependent order.
"""
from __future__ import annotations

import bisect

import torch

from .moe import RoutedMoE

DECODE_ROWS = (1, 2, 4, 8, 16, 32, 64, 128)
PREFILL_ROWS = (256, 512, 1024, 2048, 3072)


def bucket_for(rows: int, buckets=DECODE_ROWS + PREFILL_ROWS) -> int:
    """The smallest bucket holding `rows` rows."""
    b = sorted(buckets)
    if rows < 1:
        raise ValueError(f"rows must be >= 1, got {rows}")
    i = bisect.bisect_left(b, rows)
    if i == len(b):
        raise ValueError(f"{rows} rows exceed the largest bucket ({b[-1]})")
    return b[i]


class BucketedMoE:
    """One rank's routed-MoE step replayed from a CUDA graph per row bucket.

    layer: a RoutedMoE whose max_tokens covers the largest bucket.  Graphs are
    captured on first use of a bucket (or all at once by capture()); calls run
    on the current stream and return a view of the persistent output buffer,
    valid until the next call."""

    def __init__(self, layer: RoutedMoE, buckets=DECODE_ROWS + PREFILL_ROWS):
        self.layer = layer
        self.buckets = tuple(sorted(buckets))
        top = self.buckets[-1]
        if top > layer.max_tokens:
            raise ValueError(f"largest bucket {top} exceeds the layer's max_tokens "
                             f"{layer.max_tokens}")
        dev = layer.device
        self.x = torch.zeros((top, layer.cfg.hidden), dtype=torch.bfloat16, device=dev)
        self.out = torch.empty((top, layer.cfg.hidden), dtype=torch.float32, device=dev)
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self._dirty = 0  # rows of self.x written by the previous call

    def _capture(self, b: int) -> torch.cuda.CUDAGraph:
        x, out = self.x[:b], self.out[:b]
        s = torch.cuda.Stream(device=self.layer.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            # an uncaptured launch first: it sizes the bucket's workspace and
            # creates the layer's side stream outside the capture
            self.layer(x, out)
            s.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self.layer(x, out)
        torch.cuda.current_stream().wait_stream(s)
        self.graphs[b] = g
        return g

    def capture(self, buckets=None) -> None:
        """Capture the graphs of `buckets` (all buckets by default) now."""
        for b in (buckets or self.buckets):
            if b not in self.graphs:
                self._capture(b)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """x: [T, H] bf16 on the layer's device -> fp32 partial [T, H] (a view)."""
        t = x.shape[0]
        b = bucket_for(t, self.buckets)
        g = self.graphs.get(b) or self._capture(b)
        self.x[:t].copy_(x)
        if self._dirty > t:
            self.x[t:self._dirty].zero_()
        self._dirty = t
        g.replay()
        return self.out[:t]
