"""Two-GPU NCCL tests of the sharded forms with the CUDA operators as the
per-rank compute: N-sharded QuantizedLinear + all-gather, and the
expert-parallel SwitchGLU (NCCL all-to-all dispatch and combine). Both are
checked against the CPU oracle (numpy and C restatements) within the matmul
tolerance. Skipped with fewer than two GPUs."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        import datetime

        import conftest
        conftest.load_package()
        import torch.distributed as dist

        import mlx_server_runtime_b200 as mxq
        from mlx_server_runtime_b200.distributed import (ExpertParallelSwitchGLU,
                                                         ShardedQuantizedLinear)
        from gpu_util import close, rand_weights, rand_x, to_dev, to_np
        from oracle import coracle, oracle_np

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))

        # N-sharded linear: same full weights on both ranks, each keeps its rows
        rng = np.random.default_rng(5)
        N, K, M = 3000, 1024, 4
        w_np = rand_weights(rng, (N, K), "bfloat16")
        x_np = rand_x(rng, (M, K), "bfloat16")
        wq, s, b = mxq.quantize(to_dev(w_np, "bfloat16", dev), 64, 4)
        lin = ShardedQuantizedLinear.from_full(wq, s, b, group_size=64, bits=4)
        got = lin(to_dev(x_np, "bfloat16", dev))
        torch.cuda.synchronize()
        ref = oracle_np.quantized_matmul(x_np, to_np(wq), to_np(s), to_np(b), "bfloat16", 64, 4)
        close(to_np(got), ref, "bfloat16")

        # expert parallel: 8 experts, 4 per rank, top-2 routing of each rank's tokens
        E, D, I, T, k = 8, 512, 256, 24 + 8 * rank, 2
        rng = np.random.default_rng(9)
        full = []
        for n, kk in ((I, D), (I, D), (D, I)):
            w = to_dev(rand_weights(rng, (E, n, kk), "bfloat16"), "bfloat16", dev)
            full.append(mxq.quantize(w, 64, 4))
        el = E // world
        local = [tuple(a[rank * el:(rank + 1) * el].contiguous() for a in t) for t in full]
        rr = np.random.default_rng(40 + rank)
        x_np = rand_x(rr, (T, D), "bfloat16")
        idx_np = np.array([rr.choice(E, size=k, replace=False) for _ in range(T)], np.int32)
        moe = ExpertParallelSwitchGLU(*local, num_experts=E, group_size=64, bits=4)
        got = moe(to_dev(x_np, "bfloat16", dev), torch.from_numpy(idx_np).to(dev))
        torch.cuda.synchronize()
        # reference: the C oracle over the same full expert weights, per (token, expert)
        # row: silu(gate) rounded, times up rounded, then down (lfm2.py:193-218)
        host = [tuple(to_np(a) for a in t) for t in full]
        flat = idx_np.reshape(-1)
        lhs = np.repeat(np.arange(T, dtype=np.int32), k)
        xs = x_np.reshape(T, 1, D)
        g = oracle_np.to_f32(coracle.gather_qmm(xs, *host[0], flat, "bfloat16", 64, 4, lhs=lhs),
                             "bfloat16")
        u = oracle_np.to_f32(coracle.gather_qmm(xs, *host[1], flat, "bfloat16", 64, 4, lhs=lhs),
                             "bfloat16")
        act = oracle_np.round_to(g / (1.0 + np.exp(-g)), "bfloat16")
        h = oracle_np.from_f32(act * u, "bfloat16")
        ref = coracle.gather_qmm(h, *host[2], flat, "bfloat16", 64, 4).reshape(T, k, D)
        close(to_np(got), ref, "bfloat16")
        # the same with fixed-capacity buffers (no host synchronisation): 32 tokens x 2
        # experts = 64 routed rows at most
        moe_fixed = ExpertParallelSwitchGLU(*local, num_experts=E, group_size=64, bits=4,
                                            capacity=64)
        xd, idd = to_dev(x_np, "bfloat16", dev), torch.from_numpy(idx_np).to(dev)
        close(to_np(moe_fixed(xd, idd)), ref, "bfloat16")
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, True, ""))
    except Exception as e:
        q.put((rank, False, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_linear_and_expert_parallel_on_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for rank, ok, info in sorted(res):
        assert ok, f"rank {rank}: {info}"
