"""kq_linear_f32_static: the batched dp4a kernels with their scratch in a fixed
device array instead of the context's allocated buffer.  Compared with the
regular entry (kq_linear_f32, device pointers) on two calls in a row.  This
file is named to be collected last, and it also passes on its own."""
import numpy as np
import pytest

from pesti_b200 import kq, synthetic

pytestmark = pytest.mark.gpu

TOL = 1e-3
KQ_ERR_UNSUPPORTED = 2


def rel_err(y, ref):
    y = np.asarray(y, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


@pytest.fixture(scope="module")
def ctx():
    c = kq.Context(0)
    yield c
    c.close()


@pytest.mark.parametrize("qtype,n,k", [(kq.KQ_GGUF_Q4_K, 300, 4096), (kq.KQ_GGUF_Q6_K, 257, 14336),
                                       (kq.KQ_GGUF_Q4_K, 64, 16384), (kq.KQ_GGUF_Q6_K, 33, 4864)])
@pytest.mark.parametrize("m", [1, 2, 3, 4])
def test_static_scratch_matches_regular_entry(ctx, qtype, n, k, m):
    import torch
    raw = synthetic.gguf_weight(qtype, n, k, seed=n + m)
    w = kq.Weight(ctx, qtype, raw, n, k)
    x = torch.from_numpy(synthetic.activations(m, k, seed=m)).cuda()
    bias = torch.from_numpy(np.linspace(-1, 1, n).astype(np.float32)).cuda()
    ref = torch.empty((m, n), device="cuda")
    w.linear(x, m, ref, bias, device_ptrs=True, sync=True)
    outs = []
    for _ in range(2):  # two calls in a row reuse the same fixed scratch
        y = torch.full((m, n), float("nan"), device="cuda")
        w.linear_static(x, m, y, bias, sync=True)
        outs.append(y.cpu().numpy())
    r = ref.cpu().numpy()
    for y in outs:
        assert np.isfinite(y).all()
        assert rel_err(y, r) <= TOL
    assert np.array_equal(outs[0], outs[1])
    w.free()


def test_static_scratch_rejects_shapes_beyond_its_size(ctx):
    import torch
    n, k = 8, 32768  # 4 rows of 32768 activations need more than the fixed scratch
    raw = synthetic.gguf_weight(kq.KQ_GGUF_Q4_K, n, k, seed=1)
    w = kq.Weight(ctx, kq.KQ_GGUF_Q4_K, raw, n, k)
    x = torch.zeros((4, k), device="cuda")
    y = torch.zeros((4, n), device="cuda")
    before = ctx.launch_count
    with pytest.raises(kq.KqError) as e:
        w.linear_static(x, 4, y)
    assert e.value.status == KQ_ERR_UNSUPPORTED
    assert "scratch" in str(e.value)
    assert ctx.launch_count == before
    with pytest.raises(kq.KqError):
        w.linear_static(x, 5, y)  # more rows than the batched kernels serve
    w.free()


def test_static_entry_allocates_nothing_on_a_fresh_context():
    """A context that has only ever run kq_linear_f32_static grows no scratch:
    the device's free memory is the same before and after its calls, and the
    result matches the oracle.  The kernels run once first on a throwaway
    context, so the driver's one-time loading of their code is not counted."""
    import torch

    import oracle
    qtype, n, k, m = kq.KQ_GGUF_Q6_K, 257, 14336, 3
    raw = synthetic.gguf_weight(qtype, n, k, seed=5)
    x = torch.from_numpy(synthetic.activations(m, k, seed=6)).cuda()
    warm = kq.Context(0)
    ww = kq.Weight(warm, qtype, raw, n, k)
    yw = torch.empty((m, n), device="cuda")
    ww.linear_static(x, m, yw, sync=True)
    ww.free()
    warm.close()

    c = kq.Context(0)
    w = kq.Weight(c, qtype, raw, n, k)
    ys = [torch.full((m, n), float("nan"), device="cuda") for _ in range(2)]
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for y in ys:
        w.linear_static(x, m, y, sync=True)
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    ref = oracle.gguf_linear(oracle.GGUF_Q6_K, raw, n, k, x.cpu().numpy())
    for y in ys:
        assert rel_err(y.cpu().numpy(), ref) <= TOL
    assert torch.equal(ys[0], ys[1])
    w.free()
    c.close()
