"""The multi-GPU decomposition on CPU: partition helpers, and the two combines run as world_size-2 and -4 gloo ranks over
oracle outputs -- expert parallelism (own slots, zeros elsewhere, summed) and the row split (per-rank [M][N/G] blocks,
gathered and permuted) -- checked exactly against the one-device oracle. The combine arithmetic restated here is
what vkb_moe_ep / vkb_gemm_q4_tc_rowsplit do on the GPUs with NCCL."""
import os
import socket

import numpy as np
import pytest

from oracle import oracle as O


def test_expert_range_partitions():
    from vkb import dist as D
    for E, G in [(128, 1), (128, 2), (128, 8), (160, 8), (10, 4), (7, 7)]:
        seen = []
        for r in range(G):
            e0, el = D.expert_range(E, G, r)
            assert el >= 1
            seen.extend(range(e0, e0 + el))
        assert seen == list(range(E))
    with pytest.raises(ValueError):
        D.expert_range(3, 4, 0)


def test_row_range_partitions():
    from vkb import dist as D
    for N, G in [(12288, 8), (8192, 4), (8192, 2), (512, 1)]:
        rows = [D.row_range(N, G, r) for r in range(G)]
        assert rows[0][0] == 0 and all(a[0] + a[1] == b[0] for a, b in zip(rows, rows[1:]))
        assert rows[-1][0] + rows[-1][1] == N
    with pytest.raises(ValueError):
        D.row_range(1000, 3, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case():
    rng = np.random.default_rng(11)
    E, N, K, T, k = 8, 64, 256, 5, 3
    codes = rng.integers(-8, 8, size=(E, N, K)).astype(np.int8)
    scales = rng.uniform(0.004, 0.02, size=(E, N, K // 32)).astype(np.float16).view(np.uint16)
    idx = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    x = rng.uniform(-1, 1, size=(T, K)).astype(np.float16).view(np.uint16)
    wc = rng.integers(-8, 8, size=(96, K)).astype(np.int8)
    ws = rng.uniform(0.004, 0.02, size=(96, K // 32)).astype(np.float16).view(np.uint16)
    xp = rng.uniform(-1, 1, size=(7, K)).astype(np.float16).view(np.uint16)
    return codes, scales, idx, x, wc, ws, xp


def _rank_main(rank, world, port, q):
    try:
        import torch
        import torch.distributed as dist
        from vkb import dist as D
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
        codes, scales, idx, x, wc, ws, xp = _case()
        # expert parallel: this rank's experts only (slots of other experts stay zero), then sum over ranks
        e0, el = D.expert_range(codes.shape[0], world, rank)
        ref, _, local = O.moe_ref(codes[e0:e0 + el], scales[e0:e0 + el], idx, x, e0=e0)
        ref[~local] = 0.0
        t = torch.from_numpy(ref.copy())
        dist.all_reduce(t)
        moe_combined = t.numpy()
        # row split: this rank's rows, gathered, permuted
        n0, nl = D.row_range(wc.shape[0], world, rank)
        block = O.ref_value(wc[n0:n0 + nl], ws[n0:n0 + nl], xp)          # [M][nl]
        parts = [torch.zeros_like(torch.from_numpy(block)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(block.copy()))
        rows_combined = D.combine_rowsplit([p.numpy() for p in parts])
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, moe_combined, rows_combined, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, None, repr(e)))


@pytest.mark.parametrize("world", [2, 4])
def test_combines_gloo(world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, _, _, err in results:
        assert err is None, f"rank {rank}: {err}"
    codes, scales, idx, x, wc, ws, xp = _case()
    ref_full, _, _ = O.moe_ref(codes, scales, idx, x)
    rows_full = O.ref_value(wc, ws, xp)
    for rank, moe_c, rows_c, _ in results:
        assert np.array_equal(moe_c, ref_full), rank            # one non-zero contributor per slot: exact
        assert np.array_equal(rows_c, rows_full), rank


def test_combine_helpers_match_layouts():
    from vkb import dist as D
    rng = np.random.default_rng(3)
    blocks = [rng.standard_normal((4, 5)) for _ in range(3)]
    y = D.combine_rowsplit(blocks)
    for g in range(3):
        assert np.array_equal(y[:, 5 * g:5 * g + 5], blocks[g])
    a = np.zeros((2, 3, 4)); b = np.zeros((2, 3, 4))
    a[0, 1] = 1.5; b[1, 2] = -2.0
    s = D.combine_moe_slots([a, b])
    assert s[0, 1, 0] == 1.5 and s[1, 2, 3] == -2.0
