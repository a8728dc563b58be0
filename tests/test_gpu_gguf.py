"""Q4_K / Q6_K tensors read from a GGUF file and uploaded by kq_gguf_upload:
the same device weight and the same products as uploading the bytes
directly, within the linear tolerance of the oracle; other tensor types are
refused."""
import numpy as np
import pytest

import oracle
from pesti_b200 import kq, synthetic

gguf = pytest.importorskip("gguf")
pytestmark = pytest.mark.gpu

TOL = 1e-3


def test_upload_from_gguf_matches_direct_upload(gpu_ctx, tmp_path):
    q4 = synthetic.gguf_weight(kq.KQ_GGUF_Q4_K, 300, 1024, seed=5)
    q6 = synthetic.gguf_weight(kq.KQ_GGUF_Q6_K, 200, 2048, seed=6)
    path = tmp_path / "w.gguf"
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_tensor("a.weight", q4, raw_dtype=gguf.GGMLQuantizationType.Q4_K)
    w.add_tensor("b.weight", q6, raw_dtype=gguf.GGMLQuantizationType.Q6_K)
    w.add_tensor("norm.weight", np.ones(64, np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with kq.GgufFile(str(path)) as f:
        for name, raw, kt, ot, n, k in (("a.weight", q4, kq.KQ_GGUF_Q4_K, oracle.GGUF_Q4_K, 300, 1024),
                                        ("b.weight", q6, kq.KQ_GGUF_Q6_K, oracle.GGUF_Q6_K, 200, 2048)):
            wf = f.upload(gpu_ctx, name)
            assert (wf.kq_type, wf.out_features, wf.in_features) == (kt, n, k)
            wd = kq.Weight(gpu_ctx, kt, raw, n, k)
            assert np.array_equal(wf.dequant().view(np.uint32), wd.dequant().view(np.uint32))
            for m in (1, 5):
                x = synthetic.activations(m, k, seed=m)
                y = np.empty((m, n), np.float32)
                wf.linear(x, m, y)
                ref = oracle.gguf_linear(ot, raw, n, k, x)
                assert float(np.max(np.abs(y - ref)) / np.max(np.abs(ref))) <= TOL
        with pytest.raises(kq.KqError) as e:
            f.upload(gpu_ctx, "norm.weight")
        assert e.value.status == kq.KQ_ERR_UNSUPPORTED
        # the drop-in layer built from the same file
        ql = kq.QuantizedLinear.from_gguf(f, "b.weight", ctx=gpu_ctx)
        assert (ql.dtype, ql.in_features, ql.out_features) == ("Q6_K", 2048, 200)
        x = synthetic.activations(2, 2048, seed=9)
        y = ql.forward(x, 2).reshape(2, 200)
        ref = oracle.gguf_linear(oracle.GGUF_Q6_K, q6, 200, 2048, x)
        assert float(np.max(np.abs(y - ref)) / np.max(np.abs(ref))) <= TOL
