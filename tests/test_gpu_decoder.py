"""Decoder step on the GPU against the CPU restatement of pesti's decode step
(oracle/decoder_oracle.py) on small models: same weights, same KV-cache
prefix, logits within tolerance; CUDA-graph replay; tensor parallelism on 2
GPUs giving the same logits as one GPU."""
import dataclasses
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-3  # max|logit - ref| / max|ref| after two layers and the head

from pesti_b200 import decoder as dec  # noqa: E402
from pesti_b200 import kq  # noqa: E402

QWEN_TINY = dec.DecoderConfig("qwen-like-tiny", 2, 448, 7, 1, 64, 512, 300, 1e-6, 1e6, True)
LLAMA_TINY = dec.DecoderConfig("llama-like-tiny", 2, 512, 4, 2, 128, 768, 300, 1e-5, 5e5, False)
# FFN 1024: both column blocks fall on superblock edges at 2 ranks, so batch 1
# takes the column-split exchange of partials and batch 2 the column split with
# all-reduced partials (LLAMA_TINY, whose blocks do not, the row all-gathers)
LLAMA_TINY_TP = dec.DecoderConfig("llama-like-tiny-tp", 2, 512, 4, 2, 128, 1024, 300, 1e-5, 5e5, False)
# 16 query / 8 KV heads of 128 and FFN 4096: the column blocks stay on superblock
# edges up to 8 ranks (2 heads = 256 columns, FFN block 512)
LLAMA_TINY_TP8 = dec.DecoderConfig("llama-like-tiny-tp8", 2, 1024, 16, 8, 128, 4096, 300, 1e-5, 5e5, False)


def rel_err(y, ref):
    y = np.asarray(y, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def _oracle_caches(model, cfg):
    ks = [model.raw[(li, "kcache")].astype(np.float32) for li in range(cfg.layers)]
    vs = [model.raw[(li, "vcache")].astype(np.float32) for li in range(cfg.layers)]
    return ks, vs


# batch 1 runs the whole step as one persistent kernel ("b1"), or the fused
# single-token linears (RMSNorm / SwiGLU / residual inside the GEMV) one
# kernel per operation ("b1-kernels"); batch 2 the separate kernels;
# "unfused" forces the latter at batch 1
@pytest.mark.parametrize("cfg", [QWEN_TINY, LLAMA_TINY], ids=lambda c: c.name)
@pytest.mark.parametrize("mode", [dec.SWIGLU_REFERENCE, dec.SWIGLU_SILU])
@pytest.mark.parametrize("batch,fused,step", [(1, True, True), (1, True, False), (1, False, False), (2, True, False)],
                         ids=["b1", "b1-kernels", "b1-unfused", "b2"])
def test_decode_steps_match_the_restated_reference(gpu_ctx, cfg, mode, batch, fused, step):
    import torch
    from oracle import decoder_oracle
    ctx_len = 20
    model = dec.Decoder(cfg, gpu_ctx, batch, ctx_len, max_new=4, seed=5, swiglu_mode=mode, keep_raw=True,
                        fused=fused, step_kernel=step)
    assert model.step_kernel == step
    ks, vs = _oracle_caches(model, cfg)
    for step, toks in enumerate(([3, 250][:batch], [17, 9][:batch])):
        pos = ctx_len + step
        model.tokens.copy_(torch.tensor(toks, dtype=torch.int32))
        model.step(pos)
        gpu_ctx.synchronize()
        got = model.logits.cpu().numpy()
        ref = decoder_oracle.decode_step(cfg, model.raw, toks, pos, ks, vs, swiglu_mode=mode)
        assert np.isfinite(got).all()
        assert rel_err(got, ref) <= TOL, f"step {step}"
    model.close()


@pytest.mark.parametrize("batch,step", [(1, False), (1, True), (2, False)], ids=["b1", "b1-step-kernel", "b2"])
def test_decode_step_replays_from_a_cuda_graph(gpu_ctx, batch, step):
    import torch
    cfg = LLAMA_TINY
    model = dec.Decoder(cfg, gpu_ctx, batch, 20, max_new=2, seed=6, step_kernel=step)
    model.tokens.copy_(torch.tensor([1, 2][:batch], dtype=torch.int32))
    s = torch.cuda.Stream()
    gpu_ctx.set_stream(s.cuda_stream)
    try:
        with torch.cuda.stream(s):
            model.step(20)
        s.synchronize()
        eager = model.logits.clone()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            model.step(20)
        for _ in range(2):
            model.logits.zero_()
            with torch.cuda.stream(s):
                g.replay()
            s.synchronize()
            assert torch.equal(model.logits, eager)
        del g
    finally:
        gpu_ctx.set_stream(None)
    model.close()


# The benchmark's model shapes: Qwen2.5-0.5B-shaped in full (24 layers, 896
# activations on 1024-wide K-quant rows, vocab 151936, context 512) and
# Llama-3-8B-shaped at full width and vocabulary with 2 of its 32 layers
# (context 2048; the per-layer shapes are those of the 32-layer model).
LLAMA3_8B_2L = dataclasses.replace(dec.LLAMA3_8B, name="llama-3-8b-shaped-2-layers", layers=2)


@pytest.mark.parametrize("cfg,ctx_len,batch,step", [(dec.QWEN25_05B, 512, 1, True), (dec.QWEN25_05B, 512, 1, False),
                                                    (LLAMA3_8B_2L, 2048, 1, True), (LLAMA3_8B_2L, 2048, 1, False),
                                                    (LLAMA3_8B_2L, 2048, 8, False)],
                         ids=["qwen05b-full-b1", "qwen05b-full-b1-kernels", "llama8b-2layers-b1",
                              "llama8b-2layers-b1-kernels", "llama8b-2layers-b8"])
def test_full_shape_decode_step_matches_the_restated_reference(gpu_ctx, cfg, ctx_len, batch, step):
    import torch
    from oracle import decoder_oracle
    model = dec.Decoder(cfg, gpu_ctx, batch, ctx_len, max_new=2, seed=9, keep_raw=True, step_kernel=step)
    ks, vs = _oracle_caches(model, cfg)
    toks = [(1000 + 7919 * i) % cfg.vocab for i in range(batch)]
    model.tokens.copy_(torch.tensor(toks, dtype=torch.int32))
    model.step(ctx_len)
    gpu_ctx.synchronize()
    got = model.logits.cpu().numpy()
    model.close()
    ref = decoder_oracle.decode_step(cfg, model.raw, toks, ctx_len, ks, vs)
    assert got.shape == (batch, cfg.vocab)
    assert np.isfinite(got).all()
    err = rel_err(got, ref)
    assert err <= TOL, err
    # every sequence of the batch, not only the one with the largest logit
    for b in range(batch):
        assert rel_err(got[b], ref[b]) <= TOL, (b, rel_err(got[b], ref[b]))


def test_decoder_rejects_heads_that_do_not_split(gpu_ctx):
    with pytest.raises(ValueError):
        dec.Decoder(QWEN_TINY, gpu_ctx, 1, 8, world=2, rank=0)


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


def _tp_worker(rank, world, port, out_dir, cfg_names=("LLAMA_TINY", "LLAMA_TINY_TP")):
    import datetime
    import torch
    import torch.distributed as dist
    from oracle import decoder_oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    status = "ok"
    try:
        ctx = kq.Context(rank)
        for cfg in (globals()[c] for c in cfg_names):
            tp = kq.TensorParallel(ctx, world, rank, max_out_elems=dec.exchange_elems(cfg, 2))
            for batch, step in ((1, True), (1, False), (2, False)):
                model = dec.Decoder(cfg, ctx, batch, 20, max_new=3, world=world, rank=rank, tp=tp, seed=7,
                                    keep_raw=True, step_kernel=step)
                single = dec.Decoder(cfg, ctx, batch, 20, max_new=3, seed=7, step_kernel=step)
                expect_split = cfg is not LLAMA_TINY and batch == 1
                if status == "ok" and model.col_split != expect_split:
                    status = f"{cfg.name} batch {batch}: column split {model.col_split}"
                if status == "ok" and model.col_batch != (cfg is not LLAMA_TINY and batch > 1):
                    status = f"{cfg.name} batch {batch}: batched column split {model.col_batch}"
                ks, vs = _oracle_caches(model, cfg)
                for pos in (20, 21):  # two steps: the exchange slots alternate
                    toks = [4 + pos, 5][:batch]
                    for m in (model, single):
                        m.tokens.copy_(torch.tensor(toks, dtype=torch.int32))
                        m.step(pos)
                    ctx.synchronize()
                    a, b = model.logits.cpu().numpy(), single.logits.cpu().numpy()
                    ref = decoder_oracle.decode_step(cfg, model.raw, toks, pos, ks, vs)
                    # Row blocks reproduce the one-GPU sums exactly.  The column split adds each
                    # projection in per-rank parts: f32 rounding differs, and the activations'
                    # 15-bit quantization can round a value one step apart, so it is held to the
                    # oracle's tolerance and half of it against one GPU.
                    tol = TOL / 2 if model.col_split or model.col_batch else 1e-5
                    if status == "ok" and (not np.isfinite(a).all() or rel_err(a, b) > tol or rel_err(a, ref) > TOL):
                        status = (f"{cfg.name} batch {batch} step {step} pos {pos}: logits differ: {rel_err(a, b):.2e} "
                                  f"from one GPU, {rel_err(a, ref):.2e} from the oracle")
                model.close()
                single.close()
            tp.close()
        ctx.close()
    except Exception as e:
        status = f"exception: {e!r}"
    finally:
        with open(os.path.join(out_dir, f"r{rank}"), "w") as fh:
            fh.write(status)
        dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_tensor_parallel_decode_matches_one_gpu(tmp_path):
    import torch.multiprocessing as mp
    mp.start_processes(_tp_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    for r in range(2):
        assert (tmp_path / f"r{r}").read_text() == "ok", f"rank {r}"


@pytest.mark.skipif(_gpus() < 4, reason="needs 4 GPUs")
def test_tensor_parallel_decode_on_every_gpu(tmp_path):
    """4 or 8 ranks (all GPUs of the box, up to 8): column-split exchange at
    batch 1, column split with all-reduced partials at batch 2, against one
    GPU and the oracle."""
    import torch.multiprocessing as mp
    world = 8 if _gpus() >= 8 else 4
    mp.start_processes(_tp_worker, args=(world, _free_port(), str(tmp_path), ("LLAMA_TINY_TP8",)), nprocs=world,
                       start_method="spawn", join=True)
    for r in range(world):
        assert (tmp_path / f"r{r}").read_text() == "ok", f"rank {r}"
