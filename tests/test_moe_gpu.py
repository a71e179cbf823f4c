"""GPU parity of the one-launch MoE decode (vkb_moe / vkb_moe_q4) against the oracle.

The reference's MoE check gives each expert its own weights and token so a wrong expert index fails
(src/bakeoff.cu:318-369); here the index list is on the device: k distinct experts per token from a seeded draw, the
pool shapes of BASELINE's MoE configs (128 x 512x2048 with k=8 plus the 2048x512 down set, 160 x 640x2560 with k=10),
1/8/64 tokens, every output slot checked, and expert-parallel subsets: a pool holding experts [e0, e0+E_local)
writes exactly the slots routed to it and leaves the others untouched."""
import numpy as np
import pytest

import vkb
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _pool(rng, fmt, E, N, K):
    lo, hi = {O.FMT_Q4: (-8, 7), O.FMT_Q8: (-127, 127), O.FMT_Q2: (-2, 1)}[fmt]
    codes = rng.integers(lo, hi + 1, size=(E, N, K)).astype(np.int8)
    scales = rng.uniform(0.004, 0.02, size=(E, N, K // 32)).astype(np.float16).view(np.uint16)
    return codes, scales


def _upload(fmt, codes, scales, sabotage=False):
    E, N, K = codes.shape
    packed = np.stack([O.pack(fmt, codes[e], sabotage=sabotage).view(np.uint8).reshape(N, -1) for e in range(E)])
    return (vkb.to_device_packed(packed.reshape(E * N, -1)),
            vkb.to_device_f16(scales.reshape(E * N, -1)).reshape(E, N, K // 32))


def _run(fmt, q, s, idx, x, E_local=None, e0=0, sentinel=None):
    import torch
    T, k = idx.shape
    N = s.shape[1]
    y = None
    if sentinel is not None:
        y = torch.full((T, k, N), sentinel, dtype=torch.float16, device="cuda")
    y = vkb.moe(fmt, q, s, torch.from_numpy(idx).cuda(), vkb.to_device_f16(x), y=y, E_local=E_local, e0=e0)
    torch.cuda.synchronize()
    return y.float().cpu().numpy().reshape(T * k, N).astype(np.float64)


@pytest.mark.parametrize("E,N,K,k,T", [(128, 512, 2048, 8, 1), (128, 512, 2048, 8, 8), (128, 512, 2048, 8, 64),
                                       (128, 2048, 512, 8, 8), (160, 640, 2560, 10, 1), (160, 640, 2560, 10, 8)])
def test_moe_baseline_pools(cuda, E, N, K, k, T):
    rng = np.random.default_rng(E + N + T)
    codes, scales = _pool(rng, O.FMT_Q4, E, N, K)
    q, s = _upload(O.FMT_Q4, codes, scales)
    idx = vkb.synth_topk(7 + T, T, E, k)
    x = (rng.uniform(-1, 1, size=(T, K))).astype(np.float16).view(np.uint16)
    y = _run(O.FMT_Q4, q, s, idx, x)
    ref, mag, local = O.moe_ref(codes, scales, idx, x)
    assert local.all()
    err, m, n = O.check_error(y, ref, mag)
    assert err <= 1e-3, (err, m, n)
    assert O.allclose_f16out(y, ref)


@pytest.mark.parametrize("fmt", [O.FMT_Q4, O.FMT_Q8, O.FMT_Q2])
def test_moe_formats_and_crowded_expert(cuda, fmt):
    """Every format; one expert chosen by 20 tokens (more than one 8-token column group) and duplicate slots."""
    rng = np.random.default_rng(50 + fmt)
    E, N, K, T, k = 12, 160, 1024, 20, 3
    codes, scales = _pool(rng, fmt, E, N, K)
    q, s = _upload(fmt, codes, scales)
    idx = vkb.synth_topk(3, T, E, k)
    idx[:, 0] = 5          # expert 5 in every token
    idx[3, 2] = idx[3, 1]  # a duplicated expert inside one token
    x = rng.uniform(-1, 1, size=(T, K)).astype(np.float16).view(np.uint16)
    y = _run(fmt, q, s, idx, x)
    ref, mag, _ = O.moe_ref(codes, scales, idx, x)
    err, m, n = O.check_error(y, ref, mag)
    assert err <= 1e-3, (err, m, n)


@pytest.mark.parametrize("fmt", [O.FMT_Q4, O.FMT_Q8, O.FMT_Q2])
@pytest.mark.parametrize("T", [1, 3, 8])
def test_moe_few_tokens_with_repeated_experts(cuda, fmt, T):
    """At most 8 tokens (their rows stay staged, and a column finds its token as slot / k): more slots per token than
    experts, so experts repeat inside a token; token 0 sends all its slots to one expert (one 8-column group of a
    single token); ragged row tiles (N = 96 + 8)."""
    rng = np.random.default_rng(60 + 10 * fmt + T)
    E, N, K, k = 6, 104, 768, 8
    codes, scales = _pool(rng, fmt, E, N, K)
    q, s = _upload(fmt, codes, scales)
    idx = rng.integers(0, E, size=(T, k)).astype(np.int32)
    idx[0, :] = 4
    x = rng.uniform(-1, 1, size=(T, K)).astype(np.float16).view(np.uint16)
    y = _run(fmt, q, s, idx, x)
    ref, mag, _ = O.moe_ref(codes, scales, idx, x)
    err, m, n = O.check_error(y, ref, mag)
    assert err <= 1e-3, (err, m, n)


@pytest.mark.parametrize("T", [2, 8, 20])   # 16 slots (the one-slot-per-lane routing), 64 (chunked), 160 (CTA-wide)
def test_moe_expert_parallel_subsets(cuda, T):
    """Four ranks' worth of pools (32 experts each) fill disjoint slots; their union is the full result, and a pool
    never touches slots routed elsewhere (sentinels)."""
    rng = np.random.default_rng(11 + T)
    E, N, K, k, G = 128, 512, 2048, 8, 4
    codes, scales = _pool(rng, O.FMT_Q4, E, N, K)
    idx = vkb.synth_topk(99, T, E, k)
    x = rng.uniform(-1, 1, size=(T, K)).astype(np.float16).view(np.uint16)
    ref, mag, _ = O.moe_ref(codes, scales, idx, x)
    SENT = -7.0
    union = np.full((T * k, N), np.nan)
    for r in range(G):
        e0, el = r * E // G, E // G
        q, s = _upload(O.FMT_Q4, codes[e0:e0 + el], scales[e0:e0 + el])
        y = _run(O.FMT_Q4, q, s, idx, x, E_local=el, e0=e0, sentinel=SENT)
        mine = ((idx.reshape(-1) >= e0) & (idx.reshape(-1) < e0 + el))
        assert np.all(y[~mine] == SENT)
        union[mine] = y[mine]
    assert not np.isnan(union).any()
    err, m, n = O.check_error(union, ref, mag)
    assert err <= 1e-3, (err, m, n)


@pytest.mark.parametrize("T,k", [(4, 8), (11, 3), (2, 16), (16, 8), (100, 1), (43, 3)])
def test_moe_routing_boundaries(cuda, T, k):
    """32 slots (the largest list routed one slot per lane), 33 slots over 11 tokens (the smallest list the one-warp
    router takes in 32-slot chunks, with the per-segment activation rows), 16 slots over 2 tokens with experts
    repeated across and inside tokens, 128 slots (the largest chunked list), 100 one-slot tokens on 9 experts (several
    segments per expert, experts spread over all four chunks), and 129 slots (the CTA-wide routing). 64 row tiles per
    expert put these lists on the two-CTA kernel instances (the host's bound gives CTAs 4 or more tiles); the smaller
    pools of the other tests take the one-CTA instances, which route the same way."""
    rng = np.random.default_rng(70 + T * k)
    E, N, K = 9, 1024, 512
    codes, scales = _pool(rng, O.FMT_Q4, E, N, K)
    q, s = _upload(O.FMT_Q4, codes, scales)
    idx = rng.integers(0, E, size=(T, k)).astype(np.int32)
    x = rng.uniform(-1, 1, size=(T, K)).astype(np.float16).view(np.uint16)
    y = _run(O.FMT_Q4, q, s, idx, x)
    ref, mag, _ = O.moe_ref(codes, scales, idx, x)
    err, m, n = O.check_error(y, ref, mag)
    assert err <= 1e-3, (err, m, n)


@pytest.mark.parametrize("E,N,K,T,k,crowd", [(16, 1040, 512, 96, 2, True), (1000, 64, 256, 64, 8, False),
                                               (40, 520, 512, 600, 1, False)])
def test_moe_cta_routing(cuda, E, N, K, T, k, crowd):
    """Lists of more than 128 slots are routed by the whole CTA, and every CTA must build the same segments: one expert
    taking 96+ slots (past the per-slot count, the one-warp countdown), 1000 local experts (several passes of the
    expert scan), and 600 slots (more than one per thread). Every slot written (sentinels), repeat runs bit-equal."""
    rng = np.random.default_rng(E + T + k)
    codes, scales = _pool(rng, O.FMT_Q4, E, N, K)
    q, s = _upload(O.FMT_Q4, codes, scales)
    idx = vkb.synth_topk(5 + T, T, E, k)
    if crowd:
        idx[:, 0] = 3
        idx[:, 1] = np.where(idx[:, 1] == 3, 4, idx[:, 1])
    x = rng.uniform(-1, 1, size=(T, K)).astype(np.float16).view(np.uint16)
    y = _run(O.FMT_Q4, q, s, idx, x, sentinel=-7.0)
    assert not np.any(y == -7.0)
    ref, mag, _ = O.moe_ref(codes, scales, idx, x)
    err, m, n = O.check_error(y, ref, mag)
    assert err <= 1e-3, (err, m, n)
    assert np.array_equal(_run(O.FMT_Q4, q, s, idx, x), y)


def test_moe_sabotage_fails(cuda):
    rng = np.random.default_rng(13)
    E, N, K, T, k = 16, 256, 1024, 4, 4
    codes, scales = _pool(rng, O.FMT_Q4, E, N, K)
    q, s = _upload(O.FMT_Q4, codes, scales, sabotage=True)
    idx = vkb.synth_topk(5, T, E, k)
    x = rng.uniform(-1, 1, size=(T, K)).astype(np.float16).view(np.uint16)
    ref, mag, _ = O.moe_ref(codes, scales, idx, x)
    err, _, _ = O.check_error(_run(O.FMT_Q4, q, s, idx, x), ref, mag)
    assert err > 1e-2


def test_moe_wrong_expert_index_is_caught(cuda):
    """Each expert has its own weights: routing a slot to a neighbour expert must fail the check."""
    rng = np.random.default_rng(17)
    E, N, K, T, k = 16, 256, 1024, 2, 4
    codes, scales = _pool(rng, O.FMT_Q4, E, N, K)
    q, s = _upload(O.FMT_Q4, codes, scales)
    idx = vkb.synth_topk(9, T, E, k)
    x = rng.uniform(-1, 1, size=(T, K)).astype(np.float16).view(np.uint16)
    ref, mag, _ = O.moe_ref(codes, scales, idx, x)
    wrong = idx.copy()
    wrong[0, 0] = (wrong[0, 0] + 1) % E
    err, _, _ = O.check_error(_run(O.FMT_Q4, q, s, wrong, x), ref, mag)
    assert err > 1e-2
