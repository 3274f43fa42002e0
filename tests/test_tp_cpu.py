"""Tensor-parallel composition on CPU: two gloo ranks, the oracle as each
rank's GEMM, the library's shard map (mrt_shard_rows / mrt_shard_cols).

* column-parallel (fused q,k,v; gate,up): every rank computes its rows;
  gathered in part order they equal the unsharded result bit for bit;
* row-parallel (o, down): FP32 partials summed across ranks and rounded once
  equal the unsharded FP32 sum rounded, within one FP16 ulp (only the FP32
  summation order differs) and with the same error against FP64;
* vocabulary-sharded lm_head: per-rank (value, global index) pairs combined
  with the first-maximum rule give the unsharded greedy pick.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mruntime_b200 import capi
from mruntime_b200 import workloads as W
from oracle import oracle as O

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(77)
    K = 256
    x = W.to_f16_bits(rng.standard_normal((5, K), dtype=np.float32))
    parts = (96, 32, 32)  # a small fused q,k,v
    wqkv = W.to_bf16_bits(rng.standard_normal((sum(parts), K), dtype=np.float32) * np.float32(0.05))
    wo = W.to_bf16_bits(rng.standard_normal((64, K), dtype=np.float32) * np.float32(0.05))
    vocab = W.to_f16_bits(rng.standard_normal((1000, K), dtype=np.float32) * np.float32(0.05))
    return x, parts, wqkv, wo, vocab


def _worker(rank: int, port: int, out_dir: str):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        x, parts, wqkv, wo, vocab = _inputs()
        K = x.shape[1]
        # column-parallel
        ranges = capi.shard_rows(list(parts), WORLD, rank)
        rows = np.concatenate([np.arange(b, e) for b, e in ranges])
        local = O.gemm(x, O.FP16, wqkv[rows], O.BF16, trans_b=True)
        mine = torch.from_numpy(local.astype(np.int32))  # gloo has no 16-bit integer collectives
        gathered = [torch.empty_like(mine) for _ in range(WORLD)]
        dist.all_gather(gathered, mine)
        # reassemble every part in rank order
        blocks = [g.numpy().astype(np.uint16) for g in gathered]
        per_rank_sizes = [[e - b for b, e in capi.shard_rows(list(parts), WORLD, r)] for r in range(WORLD)]
        cols = []
        for p in range(len(parts)):
            for r in range(WORLD):
                off = sum(per_rank_sizes[r][:p])
                cols.append(blocks[r][:, off:off + per_rank_sizes[r][p]])
        col_result = np.concatenate(cols, axis=1)
        # row-parallel
        k0, k1 = capi.shard_cols(K, WORLD, rank)
        part = O.gemm(np.ascontiguousarray(x[:, k0:k1]), O.FP16, np.ascontiguousarray(wo[:, k0:k1]), O.BF16,
                      c_dtype=O.FP32, trans_b=True)
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t)
        row_result = O.f32_to_f16(t.numpy())
        # vocabulary-sharded greedy pick
        (vb, ve), = capi.shard_rows([vocab.shape[0]], WORLD, rank)
        logits = O.gemm(x, O.FP16, vocab[vb:ve], O.FP16, trans_b=True)
        pairs = torch.tensor([[float(W.f16_bits_to_f32(row)[O.argmax(row)]), float(O.argmax(row) + vb)]
                              for row in logits], dtype=torch.float64)
        allp = [torch.empty_like(pairs) for _ in range(WORLD)]
        dist.all_gather(allp, pairs)
        picks = []
        for m in range(x.shape[0]):
            best = None
            for r in range(WORLD):
                v, i = allp[r][m].tolist()
                if best is None or v > best[0] or (v == best[0] and i < best[1]):
                    best = (v, i)
            picks.append(int(best[1]))
        if rank == 0:
            np.savez(os.path.join(out_dir, "tp.npz"), col=col_result, row=row_result, picks=np.array(picks))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_composition_gloo(tmp_path):
    mp.start_processes(_worker, args=(_free_port(), str(tmp_path)), nprocs=WORLD, start_method="spawn", join=True)
    got = np.load(tmp_path / "tp.npz")
    x, parts, wqkv, wo, vocab = _inputs()
    np.testing.assert_array_equal(got["col"], O.gemm(x, O.FP16, wqkv, O.BF16, trans_b=True))
    full = O.gemm(x, O.FP16, wo, O.BF16, trans_b=True)
    truth = O.gemm_f64(x, wo, O.BF16)
    f_got, f_full = W.f16_bits_to_f32(got["row"]), W.f16_bits_to_f32(full)
    spacing = np.maximum(np.spacing(np.abs(f_full).astype(np.float16)).astype(np.float32), np.float32(2 ** -24))
    assert np.all(np.abs(f_got - f_full) <= spacing)
    assert O.rel_frobenius(got["row"], truth) <= O.rel_frobenius(full, truth) * 1.001
    logits = O.gemm(x, O.FP16, vocab, O.FP16, trans_b=True)
    assert list(got["picks"]) == [O.argmax(r) for r in logits]
