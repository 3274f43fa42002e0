"""Tensor parallelism on two or more GPUs through the C ABI (NCCL and the
library's own NVLink peer exchange).

Each rank uploads its shard (column-parallel fused q,k,v and vocabulary;
row-parallel o), runs its GEMM, and the collectives assemble the result:
all-gather of q,k,v columns, FP32 all-reduce + one rounding for o (NCCL, and
again through mrt_tp_gemm_rowpar's peer exchange), and the sharded greedy
pick.  Rank 0 compares with the same GEMMs on one GPU and with
the oracle.  Needs >= 2 GPUs; skipped otherwise."""
import os
import socket

import numpy as np
import pytest
import torch

from gpu_util import REF_ERR_SLACK  # noqa: E402

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    from mruntime_b200 import workloads as W

    rng = np.random.default_rng(2024)
    K = 512
    x = W.to_f16_bits(rng.standard_normal((37, K), dtype=np.float32))
    parts = (256, 64, 64)
    wqkv = W.to_bf16_bits(rng.standard_normal((sum(parts), K), dtype=np.float32) * np.float32(0.02))
    wo = W.to_bf16_bits(rng.standard_normal((384, K), dtype=np.float32) * np.float32(0.02))
    vocab = W.to_f16_bits(rng.standard_normal((5000, K), dtype=np.float32) * np.float32(0.02))
    return x, parts, wqkv, wo, vocab


def _worker(rank: int, port: int, out_dir: str):
    import datetime

    import torch.distributed as dist

    from mruntime_b200 import capi

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120))
    tp = None
    try:
        capi.init(rank)
        s = torch.cuda.current_stream().cuda_stream
        uid = [capi.TensorParallel.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        tp = capi.TensorParallel(rank, WORLD, uid[0])
        x, parts, wqkv, wo, vocab = _inputs()
        M, K = x.shape
        xd = torch.from_numpy(x.view(np.int16)).cuda()
        # column-parallel q,k,v, gathered in part-major order per rank
        ranges = capi.shard_rows(list(parts), WORLD, rank)
        wq = capi.Weight(wqkv.ctypes.data, capi.BF16, False, sum(parts), K, ranges, None, s)
        yq = torch.empty((M, wq.n), dtype=torch.int16, device="cuda")
        capi.gemm(wq, xd.data_ptr(), K, yq.data_ptr(), wq.n, M, False, s)
        gathered = torch.empty((M, wq.n * WORLD), dtype=torch.int16, device="cuda")
        tp.allgather_cols_f16(yq.data_ptr(), M, wq.n, gathered.data_ptr(), s)
        # row-parallel o
        k0, k1 = capi.shard_cols(K, WORLD, rank)
        wot = capi.Weight(wo.ctypes.data, capi.BF16, False, wo.shape[0], K, None, (k0, k1), s)
        xs = torch.from_numpy(np.ascontiguousarray(x[:, k0:k1]).view(np.int16)).cuda()
        part = torch.empty((M, wot.n), dtype=torch.float32, device="cuda")
        yo = torch.empty((M, wot.n), dtype=torch.int16, device="cuda")
        capi.gemm_f32(wot, xs.data_ptr(), k1 - k0, part.data_ptr(), wot.n, M, s)
        tp.allreduce_f32_to_f16(part.data_ptr(), yo.data_ptr(), M * wot.n, s)
        # the same row-parallel o through the NVLink peer exchange (no NCCL),
        # three calls in a row (the exchange's epochs advance), the second on
        # fewer rows and into a strided output
        tp.p2p_init(M * wot.n)
        yo_p2p = torch.empty((M, wot.n), dtype=torch.int16, device="cuda")
        yo_p2p_strided = torch.zeros((M - 5, wot.n + 8), dtype=torch.int16, device="cuda")
        tp.gemm_rowpar(wot, xs.data_ptr(), k1 - k0, M, yo_p2p.data_ptr(), wot.n, s)
        tp.gemm_rowpar(wot, xs.data_ptr(), k1 - k0, M - 5, yo_p2p_strided.data_ptr(), wot.n + 8, s)
        tp.gemm_rowpar(wot, xs.data_ptr(), k1 - k0, M, yo_p2p.data_ptr(), wot.n, s)
        capi.sync(s)
        np.save(os.path.join(out_dir, f"yo_p2p_{rank}.npy"), yo_p2p.cpu().numpy().view(np.uint16))
        np.save(os.path.join(out_dir, f"yo_p2p_strided_{rank}.npy"), yo_p2p_strided.cpu().numpy().view(np.uint16))
        # vocabulary-sharded lm_head + greedy pick
        (vb, ve), = capi.shard_rows([vocab.shape[0]], WORLD, rank)
        wv = capi.Weight(vocab.ctypes.data, capi.FP16, False, vocab.shape[0], K, [(vb, ve)], None, s)
        logits = torch.empty((M, wv.n), dtype=torch.int16, device="cuda")
        idx = torch.empty(M, dtype=torch.int64, device="cuda")
        val = torch.empty(M, dtype=torch.float32, device="cuda")
        capi.lm_head_argmax(wv, xd.data_ptr(), K, M, logits.data_ptr(), vb, idx.data_ptr(), val.data_ptr(), s)
        picks = torch.empty(M, dtype=torch.int64, device="cuda")
        tp.argmax(val.data_ptr(), idx.data_ptr(), M, picks.data_ptr(), s)
        capi.sync(s)
        if rank == 0:
            # single-GPU references on rank 0's device
            full_q = capi.Weight(wqkv.ctypes.data, capi.BF16, False, sum(parts), K, None, None, s)
            yq1 = torch.empty((M, full_q.n), dtype=torch.int16, device="cuda")
            capi.gemm(full_q, xd.data_ptr(), K, yq1.data_ptr(), full_q.n, M, False, s)
            full_o = capi.Weight(wo.ctypes.data, capi.BF16, False, wo.shape[0], K, None, None, s)
            yo1 = torch.empty((M, full_o.n), dtype=torch.int16, device="cuda")
            capi.gemm(full_o, xd.data_ptr(), K, yo1.data_ptr(), full_o.n, M, False, s)
            capi.sync(s)
            np.savez(os.path.join(out_dir, "tp_gpu.npz"), gathered=gathered.cpu().numpy().view(np.uint16),
                     yq1=yq1.cpu().numpy().view(np.uint16), yo=yo.cpu().numpy().view(np.uint16),
                     yo1=yo1.cpu().numpy().view(np.uint16), picks=picks.cpu().numpy(),
                     ranges=np.array([capi.shard_rows(list(parts), WORLD, r) for r in range(WORLD)]))
        dist.barrier()
    finally:
        if tp is not None:
            tp.destroy()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason="needs two GPUs")
def test_tensor_parallel_two_gpus(tmp_path):
    import torch.multiprocessing as mp

    from mruntime_b200 import workloads as W
    from oracle import oracle as O

    mp.start_processes(_worker, args=(_free_port(), str(tmp_path)), nprocs=WORLD, start_method="spawn", join=True)
    g = np.load(tmp_path / "tp_gpu.npz")
    x, parts, wqkv, wo, vocab = _inputs()
    # reassemble the gathered columns (rank-major blocks of part-major rows) into q,k,v order
    per_rank = g["gathered"].shape[1] // WORLD
    cols = []
    for p in range(len(parts)):
        for r in range(WORLD):
            sizes = [e - b for b, e in g["ranges"][r]]
            off = r * per_rank + sum(sizes[:p])
            cols.append(g["gathered"][:, off:off + sizes[p]])
    q_tp = np.concatenate(cols, axis=1)
    ref_q = O.gemm(x, O.FP16, wqkv, O.BF16, trans_b=True)
    truth_q = O.gemm_f64(x, wqkv, O.BF16)
    assert np.mean(q_tp == g["yq1"]) > 0.9
    assert O.rel_frobenius(q_tp, truth_q) <= O.rel_frobenius(ref_q, truth_q) * REF_ERR_SLACK
    ref_o = O.gemm(x, O.FP16, wo, O.BF16, trans_b=True)
    truth_o = O.gemm_f64(x, wo, O.BF16)
    assert np.mean(g["yo"] == g["yo1"]) > 0.9
    assert O.rel_frobenius(g["yo"], truth_o) <= O.rel_frobenius(ref_o, truth_o) * REF_ERR_SLACK
    # NVLink peer exchange: identical on every rank, the NCCL path's sum (two
    # partials: one FP32 add, order-free), strided and shorter calls agree
    p2p = [np.load(tmp_path / f"yo_p2p_{r}.npy") for r in range(WORLD)]
    strided = [np.load(tmp_path / f"yo_p2p_strided_{r}.npy") for r in range(WORLD)]
    for r in range(1, WORLD):
        np.testing.assert_array_equal(p2p[r], p2p[0])
        np.testing.assert_array_equal(strided[r], strided[0])
    np.testing.assert_array_equal(p2p[0], g["yo"])
    np.testing.assert_array_equal(strided[0][:, : g["yo"].shape[1]], g["yo"][: strided[0].shape[0]])
    assert not strided[0][:, g["yo"].shape[1]:].any()
    logits = O.gemm(x, O.FP16, vocab, O.FP16, trans_b=True)
    f = W.f16_bits_to_f32(logits)
    top2 = np.sort(f, axis=1)[:, -2:]
    decisive = (top2[:, 1] - top2[:, 0]) > 2 * 2.0 ** (np.floor(np.log2(np.abs(top2[:, 1]))) - 10)
    ref_picks = np.array([O.argmax(r) for r in logits])
    assert np.all(g["picks"][decisive] == ref_picks[decisive])


def _exchange_worker(rank: int, world: int, port: int, out_dir: str):
    """Row-parallel o through the NVLink peer exchange at `world` ranks, five
    calls in a row on two sizes."""
    import datetime

    import torch.distributed as dist

    from mruntime_b200 import capi

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    tp = None
    try:
        capi.init(rank)
        s = torch.cuda.current_stream().cuda_stream
        uid = [capi.TensorParallel.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        tp = capi.TensorParallel(rank, world, uid[0])
        x, _, _, wo, _ = _inputs()
        M, K = x.shape
        k0, k1 = capi.shard_cols(K, world, rank)
        wot = capi.Weight(wo.ctypes.data, capi.BF16, False, wo.shape[0], K, None, (k0, k1), s)
        xs = torch.from_numpy(np.ascontiguousarray(x[:, k0:k1]).view(np.int16)).cuda()
        tp.p2p_init(M * wot.n)
        y = torch.empty((M, wot.n), dtype=torch.int16, device="cuda")
        y_short = torch.empty((M - 11, wot.n), dtype=torch.int16, device="cuda")
        for i in range(5):
            if i % 2:
                tp.gemm_rowpar(wot, xs.data_ptr(), k1 - k0, M - 11, y_short.data_ptr(), wot.n, s)
            else:
                tp.gemm_rowpar(wot, xs.data_ptr(), k1 - k0, M, y.data_ptr(), wot.n, s)
        capi.sync(s)
        np.save(os.path.join(out_dir, f"y_{rank}.npy"), y.cpu().numpy().view(np.uint16))
        np.save(os.path.join(out_dir, f"ys_{rank}.npy"), y_short.cpu().numpy().view(np.uint16))
        dist.barrier()
    finally:
        if tp is not None:
            tp.destroy()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 3,
                    reason="needs three or more GPUs")
def test_peer_exchange_every_gpu(tmp_path):
    """The peer exchange on every GPU of the box (up to 8 ranks): every rank
    holds the same rows, within the tolerance of the reference's arithmetic."""
    import torch.multiprocessing as mp

    from oracle import oracle as O

    world = min(torch.cuda.device_count(), 8)
    mp.start_processes(_exchange_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    x, _, _, wo, _ = _inputs()
    ys = [np.load(tmp_path / f"y_{r}.npy") for r in range(world)]
    shorts = [np.load(tmp_path / f"ys_{r}.npy") for r in range(world)]
    for r in range(1, world):
        np.testing.assert_array_equal(ys[r], ys[0])
        np.testing.assert_array_equal(shorts[r], shorts[0])
    np.testing.assert_array_equal(shorts[0], ys[0][: shorts[0].shape[0]])
    truth = O.gemm_f64(x, wo, O.BF16)
    ref = O.gemm(x, O.FP16, wo, O.BF16, trans_b=True)
    assert O.rel_frobenius(ys[0], truth) <= O.rel_frobenius(ref, truth) * REF_ERR_SLACK
