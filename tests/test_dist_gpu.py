"""Multi-GPU parity (2+ GPUs, one process per GPU): the expert-parallel MoE (vkb_moe_ep, and vkb_moe_ep_p2p with
the combine fused into the kernel) and the row-split prompt GEMM (vkb_gemm_q4_tc_rowsplit, and
vkb_gemm_q4_tc_rowsplit_p2p with the all-gather fused into the epilogue, called directly and replayed from a CUDA
graph) against the one-GPU calls on the same inputs -- bit-identical, since every slot / row is computed by the same
kernel code and the combines only add zeros or move values -- and against the oracle; and a fused call refused on one
rank only, which must leave its peers with a status bit rather than a silent partial result. Skipped with fewer than
two GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    try:
        import torch
        import torch.distributed as dist
        import vkb
        from vkb import dist as D
        from oracle import oracle as O
        torch.cuda.set_device(rank)
        torch.cuda.set_stream(torch.cuda.Stream())
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
        comm = D.Comm.from_torch()
        dev = torch.device("cuda", rank)
        rng = np.random.default_rng(2024)
        out = []
        # ---- expert parallel MoE: fast path (K % 256 == 0) and the general kernel (K = 640) ----
        for (E, N, K, T, k) in [(16, 512, 2048, 1, 4), (16, 512, 2048, 33, 4), (8, 256, 640, 8, 3)]:
            codes = rng.integers(-8, 8, size=(E, N, K)).astype(np.int8)
            scales = rng.uniform(0.004, 0.02, size=(E, N, K // 32)).astype(np.float16).view(np.uint16)
            idx_np = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
            x_np = rng.uniform(-1, 1, size=(T, K)).astype(np.float16).view(np.uint16)
            packed = O.pack(O.FMT_Q4, codes.reshape(E * N, K))
            qfull = vkb.to_device_packed(packed, dev).view(E, N, -1)
            sfull = vkb.to_device_f16(scales, dev)
            e0, el = D.expert_range(E, world, rank)
            qloc, sloc = qfull[e0:e0 + el].contiguous(), sfull[e0:e0 + el].contiguous()
            idx = torch.from_numpy(idx_np).to(dev)
            x = vkb.to_device_f16(x_np, dev)
            for f32 in (False, True):
                y_one = vkb.moe(O.FMT_Q4, qfull, sfull, idx, x, out_f32=f32)
                y_ep = comm.moe_ep(qloc, sloc, idx, x, E_local=el, e0=e0, out_f32=f32)
                torch.cuda.synchronize()
                same = bool(torch.equal(y_one, y_ep))
                ref, mag, _ = O.moe_ref(codes, scales, idx_np, x_np)
                yd = y_ep.float().cpu().numpy().reshape(T * k, N).astype(np.float64)
                err = O.check_error(yd, ref, mag)[0]
                out.append((f"moe E{E} N{N} K{K} T{T} k{k} f32={f32}", same, err, 1e-4 if f32 else 1e-3))
        # ---- row-split prompt GEMM ----
        for (N, K, M) in [(1024, 2048, 1), (1024, 2048, 64), (2048, 2560, 512), (512, 768, 65)]:
            codes = rng.integers(-8, 8, size=(N, K)).astype(np.int8)
            scales = rng.uniform(0.004, 0.02, size=(N, K // 32)).astype(np.float16).view(np.uint16)
            x_np = rng.uniform(-1, 1, size=(M, K)).astype(np.float16).view(np.uint16)
            qfull = vkb.to_device_packed(O.pack(O.FMT_Q4, codes), dev)
            sfull = vkb.to_device_f16(scales, dev)
            n0, nl = D.row_range(N, world, rank)
            qloc, sloc = qfull[n0:n0 + nl].contiguous(), sfull[n0:n0 + nl].contiguous()
            x = vkb.to_device_f16(x_np, dev)
            for f32 in (False, True):
                y_one = vkb.gemm_tc(qfull, sfull, x, out_f32=f32)
                y_rs = comm.gemm_rowsplit(qloc, sloc, x, N, out_f32=f32)
                torch.cuda.synchronize()
                same = bool(torch.equal(y_one, y_rs))
                ref, mag = O.ref_value(codes, scales, x_np), O.ref_scale(codes, scales, x_np)
                err = O.check_error(y_rs.float().cpu().numpy().astype(np.float64), ref, mag)[0]
                out.append((f"rowsplit N{N} K{K} M{M} f32={f32}", same, err, O.TOL_FP16))
        # ---- row split with the all-gather fused into the epilogue (peer stores into a symmetric buffer) ----
        # (40960, 256, 64), (38912, 512, 512): more tiles per rank than CTAs (two accumulators / one), so CTAs push
        # earlier tiles while the dequantising warps join the last tile's epilogue; (1024, 2048, 64), (2048, 6144, 512):
        # the one-GPU plan is split-K, which every rank's part repeats (clusters pushing their token slices)
        for (N, K, M) in [(1024, 2048, 64), (2048, 2560, 512), (512, 768, 65), (40960, 256, 64), (38912, 512, 512),
                          (2048, 6144, 512)]:
            codes = rng.integers(-8, 8, size=(N, K)).astype(np.int8)
            scales = rng.uniform(0.004, 0.02, size=(N, K // 32)).astype(np.float16).view(np.uint16)
            qfull = vkb.to_device_packed(O.pack(O.FMT_Q4, codes), dev)
            sfull = vkb.to_device_f16(scales, dev)
            n0, nl = D.row_range(N, world, rank)
            qloc, sloc = qfull[n0:n0 + nl].contiguous(), sfull[n0:n0 + nl].contiguous()
            xs = [vkb.to_device_f16(rng.uniform(-1, 1, size=(M, K)).astype(np.float16).view(np.uint16), dev)
                  for _ in range(3)]
            ysym = comm.alloc((M, N), torch.float16)
            yv = ysym.tensor()
            snaps = []
            for x in xs:   # three calls in a row on one stream; each result copied out before the next call
                comm.gemm_rowsplit_p2p(qloc, sloc, x, N, ysym)
                snaps.append(yv.clone())
            torch.cuda.synchronize()
            for i, x in enumerate(xs):
                y_one = vkb.gemm_tc(qfull, sfull, x)
                torch.cuda.synchronize()
                out.append((f"rowsplit_p2p N{N} K{K} M{M} call{i}", bool(torch.equal(y_one, snaps[i])), 0.0, 1.0))
            ysym.free()
            # the same call captured once in a CUDA graph and replayed: the epochs live in device memory, so every
            # replay is a new call
            if (N, K, M) == (1024, 2048, 64):
                ysym = comm.alloc((M, N), torch.float16)
                yv = ysym.tensor()
                xg = torch.empty_like(xs[0])
                stream = torch.cuda.current_stream()
                torch.cuda.synchronize()
                epoch0 = comm.epoch()
                g = vkb.Graph(stream)
                with g:
                    comm.gemm_rowsplit_p2p(qloc, sloc, xg, N, ysym)
                snaps = []
                for x in xs:
                    xg.copy_(x)
                    g.replay()
                    snaps.append(yv.clone())
                torch.cuda.synchronize()
                del g
                # the communicator's epoch (device memory) counts the replays: each one is a new call
                out.append(("rowsplit_p2p graph epochs", comm.epoch() == epoch0 + len(xs), 0.0, 1.0))
                for i, x in enumerate(xs):
                    y_one = vkb.gemm_tc(qfull, sfull, x)
                    torch.cuda.synchronize()
                    out.append((f"rowsplit_p2p graph replay{i}", bool(torch.equal(y_one, snaps[i])), 0.0, 1.0))
                ysym.free()
        # ---- expert-parallel MoE with the combine fused into the kernel (peer stores) ----
        for (E, N, K, T, k) in [(16, 512, 2048, 1, 4), (16, 512, 2048, 33, 4), (8, 1024, 1024, 8, 2)]:
            codes = rng.integers(-8, 8, size=(E, N, K)).astype(np.int8)
            scales = rng.uniform(0.004, 0.02, size=(E, N, K // 32)).astype(np.float16).view(np.uint16)
            qfull = vkb.to_device_packed(O.pack(O.FMT_Q4, codes.reshape(E * N, K)), dev).view(E, N, -1)
            sfull = vkb.to_device_f16(scales, dev)
            e0, el = D.expert_range(E, world, rank)
            qloc, sloc = qfull[e0:e0 + el].contiguous(), sfull[e0:e0 + el].contiguous()
            for f32 in (False, True):
                ysym = comm.alloc((T, k, N), torch.float32 if f32 else torch.float16)
                yv = ysym.tensor()
                for call in range(2):
                    idx_np = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
                    idx = torch.from_numpy(idx_np).to(dev)
                    x = vkb.to_device_f16(rng.uniform(-1, 1, size=(T, K)).astype(np.float16).view(np.uint16), dev)
                    yv.fill_(float("nan"))   # a slot nobody writes stays NaN and fails the comparison
                    torch.cuda.synchronize()
                    dist.barrier()           # no peer stores into this copy before the fill is done
                    comm.moe_ep_p2p(qloc, sloc, idx, x, E_local=el, e0=e0, y_sym=ysym)
                    torch.cuda.synchronize()
                    y_one = vkb.moe(O.FMT_Q4, qfull, sfull, idx, x, out_f32=f32)
                    torch.cuda.synchronize()
                    out.append((f"moe_p2p E{E} N{N} K{K} T{T} k{k} f32={f32} call{call}",
                                bool(torch.equal(y_one, yv)), 0.0, 1.0))
                    dist.barrier()           # every rank compared before the next call's fill
                ysym.free()
        status = vkb.device_status()
        # ---- a fused call refused by the last rank only (y is not a symmetric buffer there): that rank returns
        # VKB_EINVAL and takes part in the call's numbering with its abstain kernel; every other rank's kernel ends at
        # once (well inside the 2 s bounded waits) with bit 8, a peer's part missing, not with a silent result; the
        # epochs stay aligned and the next call on every rank is bit-exact again ----
        import time
        N, K, M = 1024, 2048, 64
        codes = rng.integers(-8, 8, size=(N, K)).astype(np.int8)
        scales = rng.uniform(0.004, 0.02, size=(N, K // 32)).astype(np.float16).view(np.uint16)
        qfull = vkb.to_device_packed(O.pack(O.FMT_Q4, codes), dev)
        sfull = vkb.to_device_f16(scales, dev)
        n0, nl = D.row_range(N, world, rank)
        qloc, sloc = qfull[n0:n0 + nl].contiguous(), sfull[n0:n0 + nl].contiguous()
        x = vkb.to_device_f16(rng.uniform(-1, 1, size=(M, K)).astype(np.float16).view(np.uint16), dev)
        ysym = comm.alloc((M, N), torch.float16)
        plain = torch.empty((M, N), dtype=torch.float16, device=dev)
        torch.cuda.synchronize()
        epoch0 = comm.epoch()
        dist.barrier()
        refuser = rank == world - 1
        t0 = time.perf_counter()
        target = vkb._ptr(plain) if refuser else ysym.ptr
        rc = vkb.lib().vkb_gemm_q4_tc_rowsplit_p2p(comm._h, vkb._ptr(qloc), vkb._ptr(sloc), vkb._ptr(x), target, N, K,
                                                   M, vkb._stream())
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        bits = vkb.device_status()
        out.append(("refusal: return code", rc == (vkb.EINVAL if refuser else 0), 0.0, 1.0))
        out.append(("refusal: status bits", bits == (0 if refuser else 8), 0.0, 1.0))
        out.append(("refusal: no timeout", dt < 1.0, 0.0, 1.0))
        out.append(("refusal: epochs aligned", comm.epoch() == epoch0 + 1, 0.0, 1.0))
        dist.barrier()
        comm.gemm_rowsplit_p2p(qloc, sloc, x, N, ysym)
        y_next = ysym.tensor().clone()
        y_one = vkb.gemm_tc(qfull, sfull, x)
        torch.cuda.synchronize()
        out.append(("refusal: next call exact", bool(torch.equal(y_one, y_next)), 0.0, 1.0))
        out.append(("refusal: next call status", vkb.device_status() == 0, 0.0, 1.0))
        dist.barrier()
        ysym.free()
        comm.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, out, status, None))
    except Exception as e:
        import traceback
        q.put((rank, None, None, traceback.format_exc()))


def test_ep_and_rowsplit_match_one_gpu():
    import torch
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs at least two GPUs")
    world = min(n, 8)
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, out, status, err in results:
        assert err is None, f"rank {rank}:\n{err}"
        assert status == 0, (rank, status)
        for name, same, e, tol in out:
            assert same, f"rank {rank} {name}: differs from the one-GPU result"
            assert e <= tol, (rank, name, e)
