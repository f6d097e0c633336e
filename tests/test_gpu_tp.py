"""Tensor parallelism on 2 GPUs (one process per GPU, NCCL over NVLink).

- the communicator's all-reduce sums exactly (small integers in fp32);
- a 2-rank tensor-parallel decode (column-parallel q/k/v/gate/up,
  row-parallel o/down with the all-reduce, vocabulary-sharded lm head with
  the cross-rank argmax) gives the same 64 greedy tokens on both ranks as
  the oracle's unsharded decode of the same synthetic weights;
- a 2-rank prompt prefill followed by decode gives the oracle's tokens.

Skipped on a box with fewer than 2 GPUs. Children bind one GPU each and
run with NVLink SHARP (NVLS) off, so no rank binds memory to an NVLink
multicast object; the parent bounds every wait and kills its own children
if one stalls.
"""
import datetime
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from oracle import py_oracle as po

pytestmark = pytest.mark.gpu

TP_CFG = dict(n_layer=2, n_embd=512, n_head=4, n_head_kv=2, head_dim=128, n_ff=1024,
              vocab=2048, eps=1e-5, rope_theta=500000.0, wtype=po.Q4_0, etype=po.Q8_0)
SEED = 20261203
STEPS = 64


def _gpu_count():
    import torch
    return torch.cuda.device_count()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cfg, prompt, steps, max_ctx, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    out = {"rank": rank}
    try:
        import torch.distributed as dist
        from prosperoai_b200.api import Device, Model, Session, TPComm
        from test_gpu_model import gpu_generate
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        dev = Device(rank)
        comm = TPComm.over_group(dev, rank, world)
        n = 4096
        buf = dev.put(np.arange(n, dtype=np.float32) * (rank + 1))
        comm.allreduce(buf, n)
        dev.sync()
        out["allreduce"] = buf.download(np.float32)
        model = Model(dev, cfg, tp_rank=rank, tp_size=world)
        model.synthesize(SEED)
        model.set_tp(comm)
        sess = Session(model, 1, max_ctx)
        out["tokens"] = gpu_generate(sess, prompt, steps)
        dist.barrier()
        sess.close()
        comm.close()
        model.close()
        dev.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which fails the test
        out["error"] = repr(e)
    q.put(out)


def _prefill_worker(rank, world, port, cfg, prompt, steps, max_ctx, q):
    """Prompt prefill under tensor parallelism, then greedy decode steps."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    out = {"rank": rank}
    try:
        import torch.distributed as dist
        from prosperoai_b200.api import Device, Model, Session, TPComm
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        dev = Device(rank)
        comm = TPComm.over_group(dev, rank, world)
        model = Model(dev, cfg, tp_rank=rank, tp_size=world)
        model.synthesize(SEED)
        model.set_tp(comm)
        sess = Session(model, 1, max_ctx)
        toks = [int(sess.prefill(np.asarray(prompt, np.int32)[None, :])[0])]
        for _ in range(steps - 1):
            toks.append(int(sess.step(np.array([toks[-1]], np.int32))[0]))
        out["tokens"] = toks
        dist.barrier()
        sess.close()
        comm.close()
        model.close()
        dev.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which fails the test
        out["error"] = repr(e)
    q.put(out)


def _run_ranks(world, cfg, prompt, steps, max_ctx, target=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target or _worker, args=(r, world, port, cfg, prompt, steps, max_ctx, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r = q.get(timeout=600)
            results[r["rank"]] = r
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
                p.join()
    return results


def test_tp2_decode_matches_oracle(dev):
    if _gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    from test_gpu_model import oracle_generate, synth_weights
    cfg = dict(TP_CFG)
    prompt = list(np.random.default_rng(7).integers(0, cfg["vocab"], 5))
    max_ctx = len(prompt) + STEPS + 4
    w = synth_weights(dev, cfg, SEED)
    want, _ = oracle_generate(cfg, w, prompt, STEPS, max_ctx)
    res = _run_ranks(2, cfg, prompt, STEPS, max_ctx)
    for r in range(2):
        assert "error" not in res[r], res[r]["error"]
        np.testing.assert_array_equal(res[r]["allreduce"], np.arange(4096, dtype=np.float32) * 3)
        assert res[r]["tokens"] == [int(t) for t in want], f"rank {r}"


def test_tp2_prefill_then_decode_matches_oracle(dev):
    """Prompt prefill with 2 ranks (Q8_0 layers: the batched GEMV; the
    row-parallel outputs summed by the NCCL all-reduce), then decode: the
    tokens equal the oracle's stepped decode."""
    if _gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    from test_gpu_model import oracle_generate, synth_weights
    cfg = dict(TP_CFG, wtype=po.Q8_0)
    prompt = list(np.random.default_rng(8).integers(0, cfg["vocab"], 29))
    steps = 24
    max_ctx = len(prompt) + steps + 4
    w = synth_weights(dev, cfg, SEED)
    want, _ = oracle_generate(cfg, w, prompt, steps, max_ctx)
    res = _run_ranks(2, cfg, prompt, steps, max_ctx, target=_prefill_worker)
    for r in range(2):
        assert "error" not in res[r], res[r]["error"]
        assert res[r]["tokens"] == [int(t) for t in want], f"rank {r}"


# ---- the benchmark's 8B shape at 2, 4 and 8 ranks ----------------------------------

TP_8B = dict(n_layer=32, n_embd=4096, n_head=32, n_head_kv=8, head_dim=128, n_ff=14336,
             vocab=128256, eps=1e-5, rope_theta=500000.0, wtype=po.Q4_0, etype=po.Q8_0)
SEED_8B = 8008


@pytest.fixture(scope="module")
def oracle_8b(dev):
    """The oracle's greedy tokens for the 8B-shaped model, computed once for
    every world size (skipped without a second GPU)."""
    if _gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    from test_gpu_model import oracle_generate, synth_weights
    prompt = [int(t) for t in np.random.default_rng(SEED_8B).integers(0, TP_8B["vocab"], 4)]
    max_ctx = len(prompt) + STEPS
    w = synth_weights(dev, TP_8B, SEED_8B)
    want, _ = oracle_generate(TP_8B, w, prompt, STEPS, max_ctx, threads=max(8, os.cpu_count() or 8))
    return prompt, max_ctx, [int(t) for t in want]


def _worker_8b(rank, world, port, cfg, prompt, steps, max_ctx, q, persistent="0"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["PAI_B200_PERSISTENT"] = persistent
    out = {"rank": rank}
    try:
        import torch.distributed as dist
        from prosperoai_b200.api import Device, Model, Session, TPComm
        from test_gpu_model import gpu_generate
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        dev = Device(rank)
        comm = TPComm.over_group(dev, rank, world)
        model = Model(dev, cfg, tp_rank=rank, tp_size=world)
        model.synthesize(SEED_8B)
        model.set_tp(comm)
        sess = Session(model, 1, max_ctx)
        out["kernels"] = sess.step_kernels
        out["tokens"] = gpu_generate(sess, prompt, steps)
        dist.barrier()
        sess.close()
        comm.close()
        model.close()
        dev.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which fails the test
        out["error"] = repr(e)
    q.put(out)


def _worker_8b_persistent(rank, world, port, cfg, prompt, steps, max_ctx, q):
    _worker_8b(rank, world, port, cfg, prompt, steps, max_ctx, q, persistent="1")


@pytest.mark.parametrize("persistent", [False, True])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_8b_shape_decode_matches_oracle(oracle_8b, world, persistent):
    """Column-parallel q/k/v/gate/up, row-parallel o/down with the peer-memory
    exchange, KV cache split by KV head (one per rank at 8), vocabulary-sharded
    lm head with the cross-rank argmax: 64 greedy tokens on every rank equal
    the oracle's unsharded decode of the same weights."""
    if _gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    prompt, max_ctx, want = oracle_8b
    res = _run_ranks(world, TP_8B, prompt, STEPS, max_ctx,
                     target=_worker_8b_persistent if persistent else _worker_8b)
    for r in range(world):
        assert "error" not in res[r], res[r]["error"]
        assert (res[r]["kernels"] == 3) == persistent  # 3: layers, lm head shard, greedy pick over peer memory
        assert res[r]["tokens"] == want, f"rank {r} of {world}"


def _skip_worker(rank, world, port, cfg, prompt, steps, max_ctx, q):
    """Both ranks decode a few steps; then rank 1 skips a step (it leaves
    between steps, nothing of it in flight) while rank 0 runs one with a
    200 ms wait limit. The persistent step's exchanges are bounded peer-memory
    waits, not collective library calls, so rank 0 gets PAI_ERR_TIMEOUT and
    its session then refuses further steps."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["PAI_B200_PERSISTENT"] = "1"  # the step holds no collective library call
    out = {"rank": rank}
    try:
        import torch.distributed as dist
        from prosperoai_b200 import PaiError, _native
        from prosperoai_b200.api import Device, Model, Session, TPComm
        from test_gpu_model import gpu_generate
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        dev = Device(rank)
        comm = TPComm.over_group(dev, rank, world)
        model = Model(dev, cfg, tp_rank=rank, tp_size=world)
        model.synthesize(SEED)
        model.set_tp(comm)
        sess = Session(model, 1, max_ctx)
        out["kernels"] = sess.step_kernels
        out["tokens"] = gpu_generate(sess, prompt, steps)
        dist.barrier()
        if rank == 0:
            _native.check(_native.load().pai_b200_set_wait_limit(dev.ctx, 200_000_000), "set_wait_limit")
            try:
                sess.step(np.array([out["tokens"][-1]], np.int32))
                out["first"] = 0
            except PaiError as e:
                out["first"] = e.status
            try:
                sess.step(np.array([out["tokens"][-1]], np.int32))
                out["second"] = 0
            except PaiError as e:
                out["second"] = e.status
        dist.barrier()  # rank 1 stays idle until rank 0 is done
        sess.close()
        comm.close()
        model.close()
        dev.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which fails the test
        out["error"] = repr(e)
    q.put(out)


def test_tp2_rank_that_skips_a_step_times_out_the_other(dev):
    if _gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    cfg = dict(TP_CFG)
    prompt = [3, 1, 4]
    res = _run_ranks(2, cfg, prompt, 6, 64, target=_skip_worker)
    for r in range(2):
        assert "error" not in res[r], res[r]["error"]
        assert res[r]["kernels"] == 3  # layers, lm head shard, greedy pick over peer memory
    assert res[0]["tokens"] == res[1]["tokens"]
    assert res[0]["first"] == -5  # PAI_ERR_TIMEOUT
    assert res[0]["second"] == -8  # PAI_ERR_INIT: the session refuses further steps
