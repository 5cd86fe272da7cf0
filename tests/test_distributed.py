"""World-size-2 gloo tests (CPU) of the multi-GPU host logic: N-sharded
QuantizedLinear with an output all-gather, and the expert-parallel SwitchGLU
with count exchange, dispatch all-to-all and combine all-to-all.

The per-rank compute is the numpy oracle here, so the sharded results must equal
the unsharded oracle bit for bit (every output element is computed from the
same operands either way)."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bits(t):  # bf16 torch (CPU) -> uint16 bit pattern for the oracle
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _bf16(a):  # uint16 bit pattern -> bf16 torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def _oracle_qmm(x, w, s, b, group_size, bits, bias=None):
    from oracle import oracle_np
    y = oracle_np.quantized_matmul(_bits(x), w.numpy(), _bits(s), _bits(b), "bfloat16",
                                   group_size, bits, None if bias is None else _bits(bias))
    return _bf16(y)


def _oracle_gather(x, w, s, b, rhs, group_size, bits, sorted_indices):
    from oracle import oracle_np
    y = oracle_np.gather_qmm(_bits(x), w.numpy(), _bits(s), _bits(b), rhs.numpy(), "bfloat16",
                             group_size, bits)
    return _bf16(y)


def _setup(rank, world, port):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import conftest  # registers the package under its importable name
    conftest.load_package()
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    return dist


def _problem(seed, N, K, E=None, gs=64, bits=4):
    """Full (unsharded) packed weights from the oracle's quantizer, same on every rank."""
    from oracle import oracle_np
    rng = np.random.default_rng(seed)
    shape = (N, K) if E is None else (E, N, K)
    w = oracle_np.from_f32(rng.standard_normal(shape, dtype=np.float32) * 0.02, "bfloat16")
    wq, s, b = oracle_np.quantize(w.reshape(-1, K), "bfloat16", gs, bits)
    lead = shape[:-1]
    return (torch.from_numpy(wq).reshape(*lead, -1), _bf16(s).reshape(*lead, -1),
            _bf16(b).reshape(*lead, -1))


def _sharded_linear_worker(rank, world, port, N, K, M, use_bias, q):
    try:
        dist = _setup(rank, world, port)
        from mlx_server_runtime_b200.distributed import ShardedQuantizedLinear
        from oracle import oracle_np
        wq, s, b = _problem(11, N, K)
        rng = np.random.default_rng(12)
        x = _bf16(oracle_np.from_f32(rng.standard_normal((M, K), dtype=np.float32), "bfloat16"))
        bias = _bf16(oracle_np.from_f32(rng.standard_normal(N, dtype=np.float32), "bfloat16")) \
            if use_bias else None
        lin = ShardedQuantizedLinear.from_full(wq, s, b, bias, group_size=64, bits=4,
                                               local_qmm=_oracle_qmm)
        got = lin(x.reshape(1, M, K))
        ref = _oracle_qmm(x, wq, s, b, 64, 4, bias).reshape(1, M, N)
        ok = got.shape == ref.shape and torch.equal(got.view(torch.int16), ref.view(torch.int16))
        q.put((rank, bool(ok), tuple(got.shape)))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, False, repr(e)))


def _oracle_gather_skip_padding(x, w, s, b, rhs, group_size, bits, sorted_indices):
    """The oracle gather for rows with an expert; padding rows (rhs < 0) give zeros
    (the GPU gathers leave them unwritten)."""
    y = torch.zeros(rhs.shape[0], x.shape[1], w.shape[1], dtype=torch.bfloat16)
    keep = (rhs >= 0).nonzero().reshape(-1)
    if keep.numel():
        y[keep] = _oracle_gather(x[keep], w, s, b, rhs[keep], group_size, bits, sorted_indices)
    return y


def _ep_worker(rank, world, port, E, D, I, tokens, k, capacity, q):
    try:
        dist = _setup(rank, world, port)
        from mlx_server_runtime_b200.distributed import ExpertParallelSwitchGLU
        from oracle import oracle_np
        gate, up, down = _problem(21, I, D, E), _problem(22, I, D, E), _problem(23, D, I, E)
        el = E // world
        local = lambda t: tuple(a[rank * el:(rank + 1) * el].contiguous() for a in t)  # noqa
        rng = np.random.default_rng(30 + rank)
        T = tokens[rank]
        x = _bf16(oracle_np.from_f32(rng.standard_normal((T, D), dtype=np.float32), "bfloat16"))
        # top-k distinct experts per token; rank 1's tokens avoid expert 0 so the
        # per-destination counts are uneven
        lo = 1 if rank == 1 else 0
        idx = np.array([rng.choice(np.arange(lo, E), size=k, replace=False) for _ in range(T)],
                       dtype=np.int32).reshape(T, k)
        idx = torch.from_numpy(idx)
        moe = ExpertParallelSwitchGLU(local(gate), local(up), local(down), num_experts=E,
                                      group_size=64, bits=4, capacity=capacity,
                                      local_gather=_oracle_gather_skip_padding)
        got = moe(x, idx)
        # unsharded reference: every (token, slot) through its expert, one row at a time
        ref = torch.empty(T, k, D, dtype=torch.bfloat16)
        for t in range(T):
            for j in range(k):
                e = int(idx[t, j])
                xr = x[t:t + 1]
                g = _oracle_qmm(xr, gate[0][e], gate[1][e], gate[2][e], 64, 4)
                u = _oracle_qmm(xr, up[0][e], up[1][e], up[2][e], 64, 4)
                h = torch.nn.functional.silu(g) * u
                ref[t, j] = _oracle_qmm(h, down[0][e], down[1][e], down[2][e], 64, 4)[0]
        ok = torch.equal(got.view(torch.int16), ref.view(torch.int16))
        q.put((rank, bool(ok), tuple(got.shape)))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, False, repr(e)))


def _run(target, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    for _ in range(world):
        results.append(q.get(timeout=240))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for rank, ok, info in sorted(results):
        assert ok, f"rank {rank}: {info}"
    return results


@pytest.mark.parametrize("N,use_bias", [(384, False), (200, True), (1, False)])
def test_sharded_linear_allgather_matches_unsharded(N, use_bias):
    # 200 rows over 2 ranks leaves a ragged last shard; 1 row leaves rank 1 empty
    res = _run(_sharded_linear_worker, 2, N, 128, 3, use_bias)
    assert all(info == (1, 3, N) for _, _, info in res)


def test_expert_parallel_switchglu_matches_unsharded():
    # 4 experts over 2 ranks, rank 0 has 5 tokens and rank 1 has 3 (ragged dispatch)
    res = _run(_ep_worker, 2, 4, 64, 128, (5, 3), 2, None)
    assert sorted(info for _, _, info in res) == [(3, 2, 64), (5, 2, 64)]


def test_expert_parallel_rank_with_no_tokens():
    _run(_ep_worker, 2, 4, 64, 128, (4, 0), 2, None)


def test_expert_parallel_fixed_capacity():
    # the same exchange with fixed [world, capacity] buffers (no host synchronisation);
    # capacity above both ranks' routed rows, ragged token counts
    res = _run(_ep_worker, 2, 4, 64, 128, (5, 3), 2, 12)
    assert sorted(info for _, _, info in res) == [(3, 2, 64), (5, 2, 64)]


def test_sharded_linear_allgather_four_ranks():
    # 200 rows over 4 ranks: shards of 50, the same all-gather as at 8 GPUs
    res = _run(_sharded_linear_worker, 4, 200, 128, 3, True)
    assert all(info == (1, 3, 200) for _, _, info in res)


@pytest.mark.parametrize("capacity", [None, 24])
def test_expert_parallel_four_ranks(capacity):
    # 8 experts over 4 ranks (2 each), ragged token counts and an empty rank, both
    # exchange forms (split sizes read back, or fixed [world, capacity] buffers)
    res = _run(_ep_worker, 4, 8, 64, 128, (5, 3, 0, 6), 2, capacity)
    assert sorted(info for _, _, info in res) == [(0, 2, 64), (3, 2, 64), (5, 2, 64), (6, 2, 64)]
