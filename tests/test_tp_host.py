"""Host-side logic of the tensor-parallel linear, on CPU: row planning, the
per-shard restatement reassembling the full product, and the handle exchange
between gloo ranks (world size 2)."""
import os
import socket

import numpy as np
import pytest

import oracle
from pesti_b200 import kq, synthetic


@pytest.mark.parametrize("n", [1, 7, 896, 4096, 14336, 151936])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_rows_partition_the_weight(n, world):
    blocks = [kq.shard_rows(n, world, r) for r in range(world)]
    assert blocks[0][0] == 0 and blocks[-1][1] == n
    for (a0, a1), (b0, b1) in zip(blocks, blocks[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in blocks]
    assert max(sizes) - min(sizes) <= 1


def test_shard_rows_rejects_bad_rank():
    with pytest.raises(ValueError):
        kq.shard_rows(16, 2, 2)


@pytest.mark.parametrize("qtype,ot,k", [(kq.KQ_GGUF_Q4_K, oracle.GGUF_Q4_K, 1024),
                                        (kq.KQ_GGUF_Q6_K, oracle.GGUF_Q6_K, 1536)])
@pytest.mark.parametrize("world", [2, 4])
def test_row_shards_reassemble_the_full_product(qtype, ot, k, world):
    n, m = 40, 3
    raw = synthetic.gguf_weight(qtype, n, k, seed=3)
    x = synthetic.activations(m, k, seed=4)
    bias = np.linspace(-1, 1, n).astype(np.float32)
    full = oracle.gguf_linear(ot, raw, n, k, x, bias)
    parts = []
    for r in range(world):
        r0, r1 = kq.shard_rows(n, world, r)
        parts.append(oracle.gguf_linear(ot, raw[r0:r1], r1 - r0, k, x, bias[r0:r1]))
    assert np.array_equal(np.concatenate(parts, axis=1), full)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange_worker(rank, world, port, out_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        blobs = kq.torch_exchange(bytes([rank]) * 64)
        with open(os.path.join(out_dir, f"r{rank}"), "wb") as fh:
            fh.write(b"".join(blobs))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_between_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_exchange_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    expect = b"".join(bytes([r]) * 64 for r in range(world))
    for r in range(world):
        assert (tmp_path / f"r{r}").read_bytes() == expect
