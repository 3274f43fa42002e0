"""Back-to-back GEMMs that feed one another, with no host synchronisation.

Every tensor-core GEMM launch carries a programmatic edge to the kernel before
it in the stream: it may start while that kernel still runs, fetch its first
weight tiles early, and must wait for it before it reads activations or
writes anything.  These chains exercise both hazards that creates -- reading
an input the previous GEMM is still writing (read after write) and
overwriting a buffer the previous GEMM is still reading (write after read) --
eagerly and inside a CUDA graph, and require results bit-identical to the
same GEMMs run one at a time with a full synchronisation between them (the
kernels are deterministic: K-slices are summed in a fixed order)."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from mruntime_b200 import capi
from gpu_util import FP16, dev_u16, stream, upload

pytestmark = pytest.mark.gpu


class _View:
    """A row-major FP16 device weight used in place (mrt_weight_view)."""

    def __init__(self, t: torch.Tensor):
        self.t = t
        self.n, self.k = t.shape
        h = C.c_void_p()
        capi.call("mrt_weight_view", t.data_ptr(), self.n, self.k, C.byref(h))
        self.h = h

    def free(self):
        if self.h:
            capi.lib().mrt_weight_free(self.h)
            self.h = None


def _f16_bits(rng, shape, scale):
    return (rng.standard_normal(shape) * scale).astype(np.float16).view(np.uint16)


def _weights(rng, d_model: int, d_hidden: int, views: bool):
    shapes = [(d_hidden, d_model), (d_model, d_hidden), (d_model, d_model)]
    out = []
    for n, k in shapes:
        bits = _f16_bits(rng, (n, k), 1.0 / np.sqrt(k))
        out.append(_View(dev_u16(bits)) if views else upload(bits, FP16))
    return out


def _chain(ws, x, y1, y2, M, sync_each: bool):
    """g1: y1 = x W1^T; g2: y2 = y1 W2^T; g3: x = y2 W3^T (overwrites g1's
    input); g4: y1 = x W1^T (overwrites g2's input)."""
    w1, w2, w3 = ws
    steps = [(w1, x, y1), (w2, y1, y2), (w3, y2, x), (w1, x, y1)]
    for w, src, dst in steps:
        capi.gemm(w, src.data_ptr(), src.shape[1], dst.data_ptr(), dst.shape[1], M, False, stream())
        if sync_each:
            capi.sync(stream())


def _run(ws, x0, M, d_model, d_hidden, sync_each):
    x = x0.clone()
    y1 = torch.zeros((M, d_hidden), dtype=torch.int16, device="cuda")
    y2 = torch.zeros((M, d_model), dtype=torch.int16, device="cuda")
    _chain(ws, x, y1, y2, M, sync_each)
    capi.sync(stream())
    return x.clone(), y1.clone(), y2.clone()


# (M, d_model, d_hidden): swap-mode plans with in-kernel K-split fix-ups, and
# normal-mode plans with whole-K tiles and with a separate reduction launch.
CHAIN_SHAPES = [(1, 1024, 4096), (16, 2048, 2048), (64, 1024, 3072), (128, 1024, 2048), (512, 1536, 4096)]


@pytest.mark.parametrize("views", [False, True], ids=["tiled", "view"])
@pytest.mark.parametrize("M,d_model,d_hidden", CHAIN_SHAPES)
def test_chain_matches_serialised(cuda_dev, M, d_model, d_hidden, views):
    rng = np.random.default_rng(1000 + M + d_model + views)
    ws = _weights(rng, d_model, d_hidden, views)
    x0 = dev_u16(_f16_bits(rng, (M, d_model), 1.0))
    want = _run(ws, x0, M, d_model, d_hidden, sync_each=True)
    for _ in range(3):
        got = _run(ws, x0, M, d_model, d_hidden, sync_each=False)
        for g, w_, name in zip(got, want, ("x", "y1", "y2")):
            assert torch.equal(g, w_), f"{name} differs from the serialised chain"
    # The chain must also change the data (a no-op kernel would pass the above).
    assert not torch.equal(want[0], x0)
    for w in ws:
        w.free()


@pytest.mark.parametrize("M,d_model,d_hidden", [(1, 1024, 4096), (256, 1024, 2048)])
def test_chain_in_cuda_graph(cuda_dev, M, d_model, d_hidden):
    rng = np.random.default_rng(2000 + M)
    ws = _weights(rng, d_model, d_hidden, views=False)
    x0 = dev_u16(_f16_bits(rng, (M, d_model), 1.0))
    want = _run(ws, x0, M, d_model, d_hidden, sync_each=True)

    x = x0.clone()
    y1 = torch.zeros((M, d_hidden), dtype=torch.int16, device="cuda")
    y2 = torch.zeros((M, d_model), dtype=torch.int16, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        _chain(ws, x, y1, y2, M, sync_each=False)  # eager pass: workspace sized before capture
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        _chain(ws, x, y1, y2, M, sync_each=False)
    for _ in range(3):
        x.copy_(x0)
        y1.zero_()
        y2.zero_()
        g.replay()
        torch.cuda.synchronize()
        for got, w_, name in zip((x, y1, y2), want, ("x", "y1", "y2")):
            assert torch.equal(got, w_), f"{name} differs after graph replay"
    capi.sync(stream())
    del g
    for w in ws:
        w.free()
