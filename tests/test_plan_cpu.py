"""Host-side GEMM planner (mrt_gemm_plan, no device needed): every plan it
returns must be one the tcgen05 launcher accepts.  The same conditions are
checked by launch_tc_gemm before a launch; here they are swept over the
reference's shapes, ragged sizes and smaller SM counts on the CPU."""
from __future__ import annotations

import os

import numpy as np
import pytest

from mruntime_b200 import capi
from mruntime_b200 import workloads as W


def _shapes():
    ns = set()
    for _, n, k in W.LAYER_05B:
        ns.add((n, k))
    for _, parts, k in W.SWEEP_7B:
        ns.add((sum(parts), k))
    ns |= {(4864, 896), (151936, 896), (152064, 3584), (64, 64), (131, 896), (3581, 3576), (20000, 2048),
           (3584, 18944), (512, 70000), (40000, 4104)}
    rng = np.random.default_rng(5)
    for _ in range(20):
        ns.add((int(rng.integers(8, 40000)), int(rng.integers(1, 2400)) * 8))
    return sorted(ns)


MS = (1, 2, 4, 7, 16, 17, 32, 33, 63, 64, 65, 100, 128, 129, 300, 512, 1000, 2048, 4096)


@pytest.mark.parametrize("sms", [148, 132, 20])
def test_every_plan_is_launchable(sms):
    for N, K in _shapes():
        num_kb = -(-K // 64)
        for M in MS:
            p = capi.gemm_plan(M, N, K, sms)
            if M == 1 and 2 * N * K <= 20e6:
                # one token, a small weight: the SIMT GEMV, row quads 1/2/4/8 per CTA
                assert p["kernel"] == "gemv" and p["bn"] == 0 and p["kb_per"] == num_kb, (N, K, p)
                quads = -(-N // 4)
                assert p["grid"] in [-(-quads // rq) for rq in (1, 2, 4, 8)], (N, K, p)
                continue
            swap = M <= 64
            assert p["kernel"] == ("tcgen05-swap" if swap else "tcgen05"), (M, N, K, p)
            assert not p["cluster"]  # cluster plans need a device to check residency
            if swap:
                assert p["bn"] == (16 if M <= 16 else 32 if M <= 32 else 64), (M, p)
                tiles = -(-N // 128)
            elif p["pair"]:
                # SM pairs: 256 x 256 tiles, an even grid (two CTAs per unit at most)
                assert p["bn"] == 256 and M >= 256, (M, N, K, p)
                tiles = -(-M // 256) * -(-N // 256)
                assert p["grid"] % 2 == 0, (M, N, K, p)
            else:
                assert p["bn"] in (64, 128, 256), p
                tiles = -(-M // 128) * -(-N // p["bn"])
            full, splits, kb = p["full_tiles"], p["tail_splits"], p["kb_per"]
            assert 0 <= full <= tiles, (M, N, K, p)
            # swap-mode CTAs fit two to an SM
            assert 1 <= p["grid"] <= (2 * sms if swap else sms), (M, N, K, p)
            if swap and num_kb <= 32 * 64:
                # no swap-mode unit accumulates more than 64 k-blocks in TMEM
                assert full == 0 or num_kb <= 64, (M, N, K, p)
                assert full == tiles or kb <= 64, (M, N, K, p)
            if full < tiles:
                # Every K-slice owns at least one k-block and together they
                # cover K (otherwise an accumulator would never be written).
                assert splits >= 2 and kb >= 1, (M, N, K, p)
                assert (splits - 1) * kb < num_kb <= splits * kb, (M, N, K, p)
                units = full + (tiles - full) * splits
                assert p["grid"] <= (2 * units if p["pair"] else units), (M, N, K, p)
            else:
                assert splits == 1 and p["grid"] <= (2 * tiles if p["pair"] else tiles), (M, N, K, p)


def test_gemv_plan_rule(monkeypatch):
    """One token on a weight of at most 20 MB runs the SIMT GEMV (measured
    faster there than the swap-mode tcgen05 kernel); larger weights, and two
    or more tokens, keep the tensor cores; MRT_GEMV forces either way."""
    assert capi.gemm_plan(1, 4864, 896, 148)["kernel"] == "gemv"
    assert capi.gemm_plan(1, 896, 4864, 148)["kernel"] == "gemv"
    for N, K in ((4608, 3584), (3584, 3584), (37888, 3584), (3584, 18944), (151936, 896)):
        assert capi.gemm_plan(1, N, K, 148)["kernel"] == "tcgen05-swap", (N, K)
    assert capi.gemm_plan(2, 4864, 896, 148)["kernel"] == "tcgen05-swap"
    # enough CTAs for two per SM where the rows allow it
    assert capi.gemm_plan(1, 4864, 896, 148)["grid"] == 304
    monkeypatch.setenv("MRT_GEMV", "0")
    assert capi.gemm_plan(1, 4864, 896, 148)["kernel"] == "tcgen05-swap"
    monkeypatch.setenv("MRT_GEMV", "1")
    assert capi.gemm_plan(4, 37888, 3584, 148)["kernel"] == "gemv"
    assert capi.gemm_plan(5, 64, 64, 148)["kernel"] == "tcgen05-swap"


def test_plan_rejects_bad_shapes():
    for M, N, K in ((0, 8, 8), (1, 0, 8), (1, 8, 0), (-1, 8, 8)):
        with pytest.raises(capi.MrtError):
            capi.gemm_plan(M, N, K, 148)


def test_plan_rules_from_measurements():
    """Planner rules fitted to B200 measurements: single m-tile plans (65..128
    tokens) use 128- or 64-column tiles; SM pairs take over whole-K at a full
    last wave, K-split tails only for long K (down, K = 18944), and give way to
    the cost comparison when their last wave is nearly empty."""
    # single m-tile: never 256-column tiles
    for N, K in ((4608, 3584), (3584, 3584), (37888, 3584), (3584, 18944), (151936, 896)):
        for M in (65, 100, 128):
            assert capi.gemm_plan(M, N, K, 148)["bn"] in (64, 128), (M, N, K)
    # 7B prefill at M = 2048: pairs; whole K for q|k|v, o, gate+up; the down
    # projection's last half wave cut into K-slices
    for N, K in ((4608, 3584), (3584, 3584), (37888, 3584)):
        p = capi.gemm_plan(2048, N, K, 148)
        tiles = 8 * -(-N // 256)
        assert p["pair"] and p["full_tiles"] == tiles and p["tail_splits"] == 1, (N, K, p)
    p = capi.gemm_plan(2048, 3584, 18944, 148)
    assert p["pair"] and p["full_tiles"] == 74 and p["tail_splits"] >= 2, p
    # 76 pair tiles (a last wave of 2 on 74 pairs) at short K: not pairs
    assert not capi.gemm_plan(512, 9728, 896, 148)["pair"]
    # MRT_GEMM_PAIR_SPLITS forces the pair tail's slice count
    os.environ["MRT_GEMM_PAIR_SPLITS"] = "3"
    try:
        p = capi.gemm_plan(2048, 3584, 3584, 148)
    finally:
        os.environ.pop("MRT_GEMM_PAIR_SPLITS", None)
    assert p["pair"] and p["full_tiles"] == 74 and p["tail_splits"] == 3, p
