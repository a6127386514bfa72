"""Tensor-parallel host logic on the CPU (no GPU): the shard layout's arithmetic and the two
collective steps of the TP decode, checked with the oracle and world_size-2 gloo ranks.

The TP runner (lq_qwen3_create_tp) splits q/k/v and gate/up by output rows, o and down by K in
whole Q8_0 blocks (a row-parallel partial per rank, then a sum all-reduce), and the LM head by
vocabulary rows (argmax keys with the shard's base index, then a max all-reduce). Weights of a
shard come from the seeded generator at the full tensor's element indices."""
import os
import socket

import numpy as np
import pytest


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_generator_slices_equal_full_tensor(oracle):
    """A K-slice [rows][c0:c0+kc] generated at indices row*K + c0 + j (the 2-D fill) and a row
    range generated at offset r0*K equal the same parts of the full tensor."""
    n, k, tid, seed, std = 24, 256, 0x1234, 99, 0.02
    full = oracle.gen_bf16(seed, tid, n * k, std).reshape(n, k)
    c0, kc = 96, 64
    cols = np.stack([oracle.gen_bf16(seed, tid, kc, std, offset=r * k + c0) for r in range(n)])
    assert np.array_equal(cols, full[:, c0:c0 + kc])
    assert np.array_equal(oracle.gen_bf16(seed, tid, 5 * k, std, offset=7 * k).reshape(5, k), full[7:12])


@pytest.mark.parametrize("world", [2, 4, 8])
def test_row_parallel_partials_sum_to_full_product(oracle, rng, world):
    """o/down under TP: the K split on whole Q8_0 blocks leaves every block (and its scale)
    intact, so sum_r x_r . W_r^T is the full product up to the f32 regrouping of the block
    sum (bounded like the decode GEMV's reordering)."""
    m, n, k = 3, 64, 32 * 8 * world
    w = oracle.f32_to_bf16((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    wq, wd = oracle.q8_0_quantize(w)
    xq, xd = oracle.q8_0_quantize(rng.standard_normal((m, k)).astype(np.float32))
    full, absum = oracle.q8_0_matmul(xq, xd, wq, wd, with_abs=True)
    ks = k // world
    parts = [oracle.q8_0_matmul(np.ascontiguousarray(xq[:, r * ks:(r + 1) * ks]),
                                np.ascontiguousarray(xd[:, r * ks // 32:(r + 1) * ks // 32]),
                                np.ascontiguousarray(wq[:, r * ks:(r + 1) * ks]),
                                np.ascontiguousarray(wd[:, r * ks // 32:(r + 1) * ks // 32])) for r in range(world)]
    total = np.zeros_like(full)
    for p in parts:
        total = (total + p).astype(np.float32)
    bound = 2.0 * (k // 32 + world) * 2.0 ** -24 * absum + 1e-30
    assert np.all(np.abs(total - full) <= bound)


def _argmax_key(v: np.float32, idx: int) -> int:
    """The 64-bit argmax key: order-preserving float bits above the index (ties -> higher)."""
    b = int(np.float32(v).view(np.uint32))
    b = (b ^ 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)
    return (b << 32) | idx


def _tp_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
        from oracle import oracle as O
        rng = np.random.default_rng(5)  # same data on every rank
        m, n, k = 2, 48, 32 * 4 * world
        w = O.f32_to_bf16((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
        wq, wd = O.q8_0_quantize(w)
        xq, xd = O.q8_0_quantize(rng.standard_normal((m, k)).astype(np.float32))
        resid = rng.standard_normal((m, n)).astype(np.float32)
        ks = k // world
        sl = slice(rank * ks, (rank + 1) * ks)
        bs = slice(rank * ks // 32, (rank + 1) * ks // 32)
        part = O.q8_0_matmul(np.ascontiguousarray(xq[:, sl]), np.ascontiguousarray(xd[:, bs]),
                             np.ascontiguousarray(wq[:, sl]), np.ascontiguousarray(wd[:, bs]))
        y = torch.from_numpy((resid + part) if rank == 0 else part)  # rank 0 folds in the residual
        dist.all_reduce(y)
        full, absum = O.q8_0_matmul(xq, xd, wq, wd, with_abs=True)
        ok_sum = bool(np.all(np.abs(y.numpy() - (resid + full)) <=
                             2.0 * (k // 32 + world + 1) * 2.0 ** -24 * (absum + np.abs(resid)) + 1e-30))
        # LM head over vocabulary shards: local argmax keys, shard base added, max over ranks
        V = 40 * world
        logits = rng.standard_normal((m, V)).astype(np.float32)
        logits[1, 7] = logits[1, V - 3] = logits[1].max() + 1.0  # a tie across shards
        Vl = V // world
        keys = []
        for b in range(m):
            loc = logits[b, rank * Vl:(rank + 1) * Vl]
            keys.append(max(_argmax_key(loc[j], j) for j in range(Vl)) + rank * Vl)
        # the device reduces the keys as uint64 (NCCL); gloo's int64 max needs them shifted by
        # 2^63 so that the signed order is the unsigned one
        kt = torch.tensor([kk - (1 << 63) for kk in keys], dtype=torch.int64)
        dist.all_reduce(kt, op=dist.ReduceOp.MAX)
        tok = [(int(v) + (1 << 63)) & 0xFFFFFFFF for v in kt.tolist()]
        want = [int(O.argmax(logits[b])) for b in range(m)]
        q.put((rank, ok_sum, tok, want))
    finally:
        dist.destroy_process_group()


def test_tp_collectives_gloo_world2():
    """world_size-2 gloo ranks on the CPU run the TP decode's two collective steps with the
    oracle: the row-parallel partial sum (rank 0 adds the residual) equals the full product
    within the reorder bound, and the shard-based argmax keys reduced by max pick the global
    greedy token with ties to the highest index (the reference's rule)."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok_sum, tok, want in res:
        assert ok_sum, rank
        assert tok == want, (rank, tok, want)
        assert want[1] == 40 * 2 - 3  # the tie went to the higher index


def _ep_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
        from oracle import oracle as O
        rng = np.random.default_rng(9)  # same weights and tokens on every rank
        rows, H, E, K, I = 7, 256, 8, 2, 256

        def q8(n, k):
            return (rng.integers(-127, 128, size=(n, k), dtype=np.int8),
                    rng.integers(0x1400, 0x2000, size=(n, k // 32)).astype(np.uint16))

        xb = O.f32_to_bf16(rng.standard_normal((rows, H)).astype(np.float32))
        router = q8(E, H)
        gate = [q8(I, H) for _ in range(E)]
        up = [q8(I, H) for _ in range(E)]
        down = [q8(H, I) for _ in range(E)]
        full, ids, _ = O.moe_forward(xb, router, gate, up, down, K)
        # this rank's experts only: the others contribute zero (routing is unchanged)
        El = E // world
        zero = lambda w: (np.zeros_like(w[0]), np.zeros_like(w[1]))
        mine = lambda lst: [w if rank * El <= e < (rank + 1) * El else zero(w) for e, w in enumerate(lst)]
        part, ids_r, _ = O.moe_forward(xb, router, mine(gate), mine(up), mine(down), K)
        t = torch.from_numpy(part)
        dist.all_reduce(t)
        scale = float(np.max(np.abs(full)))
        q.put((rank, bool(np.array_equal(ids, ids_r)), float(np.max(np.abs(t.numpy() - full)) / scale)))
    finally:
        dist.destroy_process_group()


def test_ep_combine_gloo_world2():
    """Expert parallelism on world_size-2 gloo ranks with the oracle: with the router
    replicated every rank routes identically; each rank adds only its experts'
    contributions and a sum all-reduce recovers the full MoE layer up to the regrouping of
    the f32 expert sum."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, same_ids, rel in res:
        assert same_ids, rank
        assert rel <= 1e-6, (rank, rel)
