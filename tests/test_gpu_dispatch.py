"""A dispatch-shaped caller of the library.

pesti-runner's GPU linear route is LinearDispatch::forward ->
DispatchContext::dispatch_linear (pesti-runner/src/kernel/dispatch.rs:340-400,
573-591): per call it converts x to f16 on the host, transposes the f16 weight
on the host, runs a candle GEMM with host<->device copies, and adds the bias on
the host.  Its replacement keeps each layer's K-quant bytes resident in HBM
and makes one kq_linear_f32(KQ_DEVICE_PTRS) call per layer on the caller's
stream, the output of one layer feeding the next.  This file drives a
multi-layer sequence of such calls and checks that, after kq_ctx_reserve:

* nothing is allocated and nothing is copied between host and device: the
  device's free memory does not move, and the sequence captured into a CUDA
  graph holds kernel nodes only (no memcpy, memset, host or allocation node);
* every layer's output matches the oracle on that layer's actual input;
* the captured graph replays bit-identically to the eager calls.
"""
import ctypes

import numpy as np
import pytest

import oracle
from pesti_b200 import kq, synthetic

pytestmark = pytest.mark.gpu

TOL = 1e-3
_ORACLE = {kq.KQ_GGUF_Q4_K: oracle.GGUF_Q4_K, kq.KQ_GGUF_Q6_K: oracle.GGUF_Q6_K}

# (type, out_features, in_features, bias): a chain 4096 -> 1024 -> 2048 ->
# 4096 -> 512 -> 14336 with both K-quant types, with and without bias
LAYERS = [
    (kq.KQ_GGUF_Q4_K, 1024, 4096, True),
    (kq.KQ_GGUF_Q4_K, 2048, 1024, False),
    (kq.KQ_GGUF_Q6_K, 4096, 2048, True),
    (kq.KQ_GGUF_Q4_K, 512, 4096, False),
    (kq.KQ_GGUF_Q6_K, 14336, 512, True),
]


class LinearDispatch:
    """One layer as a device-resident dispatch caller holds it: the weight in
    HBM, an optional device bias, and forward() = one kq_linear_f32 call with
    device pointers on the context's (the caller's) stream."""

    def __init__(self, ctx, qtype, raw, n, k, bias):
        import torch
        self.ctx, self.n, self.k, self.qtype, self.raw = ctx, n, k, qtype, raw
        self.weight = kq.Weight(ctx, qtype, raw, n, k)
        self.bias_h = bias
        self.bias = None if bias is None else torch.from_numpy(bias).cuda()

    def forward(self, x, m, y, ctx=None):
        ctx = ctx or self.ctx
        rc = ctx.lib.kq_linear_f32(ctx.handle, self.weight.handle, ctypes.c_void_p(x.data_ptr()), m,
                                   None if self.bias is None else ctypes.c_void_p(self.bias.data_ptr()),
                                   ctypes.c_void_p(y.data_ptr()), kq.KQ_DEVICE_PTRS)
        ctx.check(rc, "kq_linear_f32")


def _graph_node_types(graph):
    from cuda.bindings import runtime as rt
    g = rt.cudaGraph_t(init_value=graph.raw_cuda_graph())
    err, _, count = rt.cudaGraphGetNodes(g, 0)  # the node count
    assert err == rt.cudaError_t.cudaSuccess
    err, nodes, count = rt.cudaGraphGetNodes(g, count)
    assert err == rt.cudaError_t.cudaSuccess
    types = []
    for node in nodes[:count]:
        err, t = rt.cudaGraphNodeGetType(node)
        assert err == rt.cudaError_t.cudaSuccess
        types.append(t)
    return types


@pytest.mark.parametrize("m", [1, 4, 16, 48])
def test_dispatch_sequence_on_a_caller_stream(m):
    import torch
    from cuda.bindings import runtime as rt
    ctx = kq.Context(0)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    rng = np.random.default_rng(m)
    layers = []
    for i, (qt, n, k, has_bias) in enumerate(LAYERS):
        raw = synthetic.gguf_weight(qt, n, k, seed=100 * m + i)
        bias = rng.standard_normal(n).astype(np.float32) if has_bias else None
        layers.append(LinearDispatch(ctx, qt, raw, n, k, bias))
        ctx.reserve(layers[-1].weight, m)
    # activations: x, then each layer's output (allocated before the calls)
    acts = [torch.from_numpy(synthetic.activations(m, LAYERS[0][2], seed=m)).cuda()]
    acts += [torch.empty((m, n), device="cuda") for _, n, _, _ in LAYERS]

    def sequence(c=None):
        for i, layer in enumerate(layers):
            layer.forward(acts[i], m, acts[i + 1], c)

    # The kernels run once first from a throwaway context (weights serve any
    # context on their device), so the driver's one-time loading of their
    # code is not counted as an allocation of the measured context.
    warm = kq.Context(0)
    for layer in layers:
        warm.reserve(layer.weight, m)
    sequence(warm)
    warm.close()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    launches0 = ctx.launch_count
    with torch.cuda.stream(stream):
        sequence()
    stream.synchronize()
    eager_launches = ctx.launch_count - launches0
    assert torch.cuda.mem_get_info()[0] == free0, "a call allocated device memory after kq_ctx_reserve"
    eager = [a.clone() for a in acts[1:]]

    # every layer against the oracle on the input that layer actually saw
    for i, layer in enumerate(layers):
        xin = acts[i].cpu().numpy()
        ref = oracle.gguf_linear(_ORACLE[layer.qtype], layer.raw, layer.n, layer.k, xin, bias=layer.bias_h)
        y = eager[i].cpu().numpy()
        err = float(np.max(np.abs(y.astype(np.float64) - ref)) / max(np.max(np.abs(ref)), 1e-30))
        assert err <= TOL, (i, err)

    # the same sequence captured on the caller's stream: kernel nodes only
    g = torch.cuda.CUDAGraph(keep_graph=True)
    launches0 = ctx.launch_count
    with torch.cuda.graph(g, stream=stream):
        sequence()
    assert ctx.launch_count - launches0 == eager_launches
    types = _graph_node_types(g)
    kernel = rt.cudaGraphNodeType.cudaGraphNodeTypeKernel
    assert types.count(kernel) == eager_launches
    assert all(t in (kernel, rt.cudaGraphNodeType.cudaGraphNodeTypeEmpty) for t in types), types
    g.instantiate()
    for _ in range(2):
        for a in acts[1:]:
            a.fill_(float("nan"))
        with torch.cuda.stream(stream):
            g.replay()
        stream.synchronize()
        for a, e in zip(acts[1:], eager):
            assert torch.equal(a, e)
    del g
    ctx.set_stream(None)
    for layer in layers:
        layer.weight.free()
    ctx.close()
