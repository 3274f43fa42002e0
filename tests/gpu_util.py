"""Helpers for the GPU parity tests: device copies of uint16 bit arrays,
calls through the C ABI, and the tolerance checks against the oracle and the
FP64 ground truth."""
from __future__ import annotations

import numpy as np
import torch

from mruntime_b200 import capi
from mruntime_b200 import workloads as W

FP16, BF16, FP32 = capi.FP16, capi.BF16, capi.FP32

# Tolerances of the linear-layer path: relative Frobenius error against FP64 at
# most 1e-3, and never worse than the reference's own error against the same
# ground truth.  "Never worse" allows 0.1% relative slack for the different
# FP32 summation order, which moves an occasional output across an FP16
# rounding midpoint in either direction (measured spread of err / ref_err over
# every workload: about +-0.03%).
REL_FROB_MAX = 1e-3
REF_ERR_SLACK = 1.001

# (what, err, ref_err) of every check_close with a reference error; written
# out at the end of the session when MRT_ERR_LOG names a file.
ERR_RATIOS: list[tuple[str, float, float]] = []


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def dev_u16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).cuda()


def host_u16(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(np.uint16)


def upload(w: np.ndarray, dtype: int, row_ranges=None, k_range=None, on_device: bool = True) -> capi.Weight:
    N, K = w.shape
    if on_device:
        src = dev_u16(w) if dtype != FP32 else torch.from_numpy(np.ascontiguousarray(w, np.float32)).cuda()
        wt = capi.Weight(src.data_ptr(), dtype, True, N, K, row_ranges, k_range, stream())
        torch.cuda.synchronize()
        del src
        return wt
    arr = np.ascontiguousarray(w)
    return capi.Weight(arr.ctypes.data, dtype, False, N, K, row_ranges, k_range, stream())


def gemm(wt: capi.Weight, x: np.ndarray | torch.Tensor, bias: bool = False) -> np.ndarray:
    xd = x if isinstance(x, torch.Tensor) else dev_u16(x)
    M = xd.shape[0]
    y = torch.empty((M, wt.n), dtype=torch.int16, device="cuda")
    capi.gemm(wt, xd.data_ptr(), xd.shape[1], y.data_ptr(), wt.n, M, bias, stream())
    capi.sync(stream())
    return host_u16(y)


def f64_truth(x: np.ndarray, w: np.ndarray, w_dtype: int, bias: np.ndarray | None = None) -> np.ndarray:
    """FP64 ground truth, computed on the GPU in float64."""
    xf = torch.from_numpy(W.f16_bits_to_f32(x)).cuda().double()
    wf32 = W.f16_bits_to_f32(w) if w_dtype == FP16 else (W.bf16_bits_to_f32(w) if w_dtype == BF16 else w)
    wf = torch.from_numpy(np.ascontiguousarray(wf32, np.float32)).cuda().double()
    y = xf @ wf.T
    if bias is not None:
        y = y + torch.from_numpy(W.bf16_bits_to_f32(bias)).cuda().double()[None, :]
    return y.cpu().numpy()


def rel_frob(got_f16: np.ndarray, truth: np.ndarray) -> float:
    g = W.f16_bits_to_f32(got_f16).astype(np.float64)
    return float(np.linalg.norm(g - truth) / np.linalg.norm(truth))


def abs_dot(x: np.ndarray, w: np.ndarray, w_dtype: int) -> np.ndarray:
    """sum_k |x_mk * w_nk| in float64 (the scale of FP32 summation error)."""
    xf = torch.from_numpy(W.f16_bits_to_f32(x)).cuda().double().abs()
    wf32 = W.f16_bits_to_f32(w) if w_dtype == FP16 else W.bf16_bits_to_f32(w)
    wf = torch.from_numpy(np.ascontiguousarray(wf32, np.float32)).cuda().double().abs()
    return (xf @ wf.T).cpu().numpy()


def check_close(got_f16: np.ndarray, truth: np.ndarray, ref_err: float | None = None, what: str = "",
                absdot: np.ndarray | None = None, K: int = 0, pre_round: np.ndarray | None = None) -> float:
    """Element-wise bound plus the Frobenius bars.

    Element bound: half an FP16 ulp of the truth (the output rounding, taken
    as 2^-10 |t| so it covers subnormal spacing too), plus half an ulp of the
    pre-bias accumulator when the output was rounded twice (``pre_round``),
    plus 4 sqrt(K) 2^-24 sum_k|x w| for FP32 summation in any order
    (``absdot``), plus the smallest FP16 subnormal."""
    g = W.f16_bits_to_f32(got_f16).astype(np.float64)
    bound = 2.0 ** -10 * np.abs(truth) + 2.0 ** -24
    if pre_round is not None:
        bound = bound + 2.0 ** -11 * np.abs(pre_round)
    if absdot is not None:
        bound = bound + 4.0 * np.sqrt(max(K, 1)) * 2.0 ** -24 * absdot
    bad = np.abs(g - truth) > bound
    assert not bad.any(), f"{what}: {int(bad.sum())} elements outside the FP16 rounding bound"
    err = rel_frob(got_f16, truth)
    assert err <= REL_FROB_MAX, f"{what}: rel Frobenius {err:.3e} > {REL_FROB_MAX}"
    if ref_err is not None:
        ERR_RATIOS.append((what, err, ref_err))
        assert err <= ref_err * REF_ERR_SLACK, f"{what}: rel Frobenius {err:.4e} worse than reference {ref_err:.4e}"
    return err


def same_fraction(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.mean(a == b))


def check_greedy_tokens(got, golden: dict, what: str) -> int:
    """Greedy tokens against the reference engine's golden.

    Every token must equal the reference's, except that the sequences may
    part at a step where the reference's two best logits are a tie at FP16
    resolution (top-2 margin at most one FP16 ulp of the best logit): there
    the order of the FP32 sums (the reference's sequential loop against the
    tensor cores' blocked one, in every layer before) decides, and the pick
    must be the reference's runner-up.  After such a step the two sequences
    continue different prefixes and are not compared.  Returns the number of
    leading tokens that are equal."""
    ref = [int(t) for t in golden["tokens"]]
    got = [int(t) for t in got]
    assert len(got) == len(ref), f"{what}: {len(got)} tokens, reference {len(ref)}"
    t = next((i for i, (a, b) in enumerate(zip(got, ref)) if a != b), None)
    if t is None:
        print(f"{what}: all {len(ref)} tokens equal to the reference engine's")
        return len(ref)
    margins, top1, runner = golden.get("margins"), golden.get("top1"), golden.get("runner_up")
    assert margins and top1 and runner, f"{what}: token {t} is {got[t]}, reference {ref[t]} (no margins recorded)"
    ulp = float(np.spacing(np.float16(abs(top1[t]))))
    assert margins[t] <= ulp, (f"{what}: token {t} is {got[t]}, reference {ref[t]}, whose top-2 margin "
                               f"{margins[t]} exceeds one FP16 ulp ({ulp}) of its best logit {top1[t]}")
    assert got[t] == runner[t], f"{what}: at the tie of step {t} picked {got[t]}, not the runner-up {runner[t]}"
    print(f"{what}: tokens 0..{t - 1} equal to the reference engine's; step {t} is a tie at FP16 resolution "
          f"(reference best {top1[t]}, runner-up {runner[t]} {margins[t]} below = one ulp) and the runner-up was "
          f"picked; the sequences then continue different prefixes")
    return t
