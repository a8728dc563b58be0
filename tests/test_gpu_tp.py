"""Tensor-parallel linear on 2+ GPUs of one node (one process per GPU): row
shards all-gathered over NVLink peer memory, and the all-reduce of per-rank
partials.  Skipped with fewer than 2 GPUs.
Each rank compares the gathered output with the unsharded product on its own
GPU (bit-identical for the row-local single-token kernel) and with the oracle."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rel_err(y, ref):
    y = np.asarray(y, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def _worker(rank, world, port, out_dir, mode):
    import datetime
    import torch
    import torch.distributed as dist
    import oracle
    from pesti_b200 import kq, synthetic
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    status = "ok"
    try:
        ctx = kq.Context(rank)
        tp = kq.TensorParallel(ctx, world, rank, max_out_elems=8 * 14336)
        if mode == "linear":
            cases = [(kq.KQ_GGUF_Q6_K, oracle.GGUF_Q6_K, 4096, 14336, 1),
                     (kq.KQ_GGUF_Q4_K, oracle.GGUF_Q4_K, 14336, 4096, 1),
                     (kq.KQ_GGUF_Q4_K, oracle.GGUF_Q4_K, 1000, 2048, 3),
                     (kq.KQ_GGUF_Q6_K, oracle.GGUF_Q6_K, 896, 4864, 8)]
            for qt, ot, n, k, m in cases:
                raw = synthetic.gguf_weight(qt, n, k, seed=n + k)
                r0, r1 = kq.shard_rows(n, world, rank)
                shard = kq.Weight(ctx, qt, np.ascontiguousarray(raw[r0:r1]), r1 - r0, k)
                full = kq.Weight(ctx, qt, raw, n, k)
                bias = np.linspace(-1, 1, n).astype(np.float32)
                bias_d = torch.from_numpy(bias).cuda()
                bias_shard = bias_d[r0:r1].contiguous()
                for call in range(3):  # consecutive calls cycle both exchange slots
                    x = synthetic.activations(m, k, seed=10 * call + m)
                    xd = torch.from_numpy(x).cuda()
                    y = torch.full((m, n), float("nan"), device="cuda")
                    tp.linear(shard, r0, n, xd, m, y, bias_shard, sync=True)
                    y_ref = torch.empty((m, n), device="cuda")
                    full.linear(xd, m, y_ref, bias_d, device_ptrs=True, sync=True)
                    yh, yr = y.cpu().numpy(), y_ref.cpu().numpy()
                    if m == 1 and not np.array_equal(yh, yr):
                        status = f"m=1 not bit-identical to the unsharded product ({n}x{k} call {call})"
                    ref = oracle.gguf_linear(ot, raw, n, k, x, bias)
                    if not np.isfinite(yh).all() or rel_err(yh, ref) > TOL:
                        status = f"{n}x{k} m={m} call {call}: error {rel_err(yh, ref):.2e}"
                shard.free()
                full.free()
        elif mode == "allreduce":
            # every rank's partial summed in rank order: the same f32 additions
            # as a sequential sum, so bit-identical to numpy's and across ranks
            m, n, ld = 5, 2800, 2816
            for call in range(3):  # consecutive calls cycle both exchange slots
                parts = [np.random.default_rng(100 * call + r).standard_normal((m, n)).astype(np.float32)
                         for r in range(world)]
                want = np.zeros((m, n), np.float32)
                for p in parts:
                    want = want + p
                pd = torch.from_numpy(parts[rank]).cuda()
                y = torch.full((m, ld), 3.0, device="cuda")
                tp.allreduce(pd, m, n, y, y_ld=ld, sync=True)
                got = y.cpu().numpy()
                if not np.array_equal(got[:, :n], want) or not (got[:, n:] == 3.0).all():
                    status = f"all-reduce call {call}: not the rank-ordered sum"
                tp.allreduce(pd, m, n, y, y_ld=ld, accumulate=True, sync=True)
                if not np.array_equal(y.cpu().numpy()[:, :n], want + want):
                    status = f"accumulating all-reduce call {call}: wrong"
        elif mode == "missing_peer":
            # the last rank never joins the call: every other rank's bounded
            # wait for its flag must give up and report an error
            n, k = 4096, 4096
            raw = synthetic.gguf_weight(kq.KQ_GGUF_Q4_K, n, k, seed=1)
            r0, r1 = kq.shard_rows(n, world, rank)
            shard = kq.Weight(ctx, kq.KQ_GGUF_Q4_K, np.ascontiguousarray(raw[r0:r1]), r1 - r0, k)
            xd = torch.ones((1, k), device="cuda")
            y = torch.empty((1, n), device="cuda")
            if rank != world - 1:
                try:
                    tp.linear(shard, r0, n, xd, 1, y, sync=True)
                    status = "the wait did not give up"
                except kq.KqError as e:
                    if "gave up" not in str(e):
                        status = f"unexpected error: {e}"
            dist.barrier()
            shard.free()
        tp.close()
        ctx.close()
    except Exception as e:  # report to the parent
        status = f"exception: {e!r}"
    finally:
        with open(os.path.join(out_dir, f"r{rank}"), "w") as fh:
            fh.write(status)
        dist.destroy_process_group()


def _run(world, mode, tmp_path):
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), mode), nprocs=world,
                       start_method="spawn", join=True)
    for r in range(world):
        assert (tmp_path / f"r{r}").read_text() == "ok", f"rank {r}"


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_tp_linear_matches_unsharded_product_2gpu(tmp_path):
    _run(2, "linear", tmp_path)


@pytest.mark.skipif(_gpus() < 4, reason="needs 4 GPUs")
def test_tp_linear_matches_unsharded_product_4gpu(tmp_path):
    _run(4, "linear", tmp_path)


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_tp_allreduce_is_the_rank_ordered_sum_2gpu(tmp_path):
    _run(2, "allreduce", tmp_path)


@pytest.mark.skipif(_gpus() < 4, reason="needs 4 GPUs")
def test_tp_allreduce_is_the_rank_ordered_sum_4gpu(tmp_path):
    _run(4, "allreduce", tmp_path)


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_tp_missing_peer_is_reported_not_hung(tmp_path):
    _run(2, "missing_peer", tmp_path)
