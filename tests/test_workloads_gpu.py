"""GPU parity at the benchmark workloads' full sizes, against golden vectors
made by the reference's own CPU gemm (tests/golden/gen_golden.py) and the FP64
ground truth.  Sizes: the Qwen2.5-0.5B decode GEMV, one 0.5B layer's
projections at M=512, the tied 0.5B lm_head with greedy argmax, and the
Qwen2.5-7B projection sweep M = 1 .. 2048."""
import hashlib

import numpy as np
import pytest
import torch

from conftest import golden
from gpu_util import (BF16, FP16, abs_dot, check_close, dev_u16, f64_truth, gemm, host_u16, rel_frob, stream,
                      upload)
from mruntime_b200 import capi
from mruntime_b200 import workloads as W

pytestmark = pytest.mark.gpu


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def test_decode_gemv_config(cuda_dev):
    g = golden("decode_gemv.npz")
    d = W.decode_gemv()
    assert sha(d["x"], d["w"]) == str(g["input_sha"]), "input generator changed"
    y = gemm(upload(d["w"], FP16), d["x"])
    err = check_close(y, g["y_f64"], float(g["ref_err"]), "decode gemv", absdot=abs_dot(d["x"], d["w"], FP16), K=896)
    print(f"decode gemv rel err {err:.4e} (reference {float(g['ref_err']):.4e}), "
          f"bit-identical to reference: {np.mean(y == g['y_ref']):.4f}")


@pytest.fixture(scope="module")
def layer():
    d = W.layer_prefill_05b()
    g = golden("layer_prefill_05b.npz")
    assert sha(*[d[k] for k in sorted(d)]) == str(g["input_sha"]), "input generator changed"
    return d, g


@pytest.mark.parametrize("name", [n for n, _, _ in W.LAYER_05B])
def test_layer_prefill_05b(cuda_dev, layer, name):
    d, g = layer
    x = d["x_down"] if name == "down" else d["x"]
    wt = upload(d[name], BF16)
    bias = None
    if name in ("q", "k", "v"):
        bias = d["b" + name]
        bd = dev_u16(bias)
        wt.attach_bias(bd.data_ptr(), BF16, True, stream())
        torch.cuda.synchronize()
    y = gemm(wt, x, bias=bias is not None)
    truth = f64_truth(x, d[name], BF16, bias=bias)
    err = check_close(y, truth, float(g[f"{name}_ref_err"]), f"layer {name}", absdot=abs_dot(x, d[name], BF16),
                      K=x.shape[1], pre_round=f64_truth(x, d[name], BF16) if bias is not None else None)
    rows = g["rows"]
    same = np.mean(y[rows] == g[f"{name}_rows"])
    assert same > 0.9
    print(f"{name}: rel err {err:.4e} reference {float(g[f'{name}_ref_err']):.4e} same-bits {same:.4f}")


@pytest.fixture(scope="module")
def lm_head():
    d = W.lm_head_05b()
    g = golden("lm_head_05b.npz")
    assert sha(d["x"], d["w"]) == str(g["input_sha"]), "input generator changed"
    return d, g


@pytest.mark.parametrize("M", [1, 128])
def test_lm_head_argmax(cuda_dev, lm_head, M):
    d, g = lm_head
    wt = upload(d["w"], FP16)
    x = dev_u16(d["x"][:M])
    V = wt.n
    logits = torch.empty((M, V), dtype=torch.int16, device="cuda")
    idx = torch.empty(M, dtype=torch.int64, device="cuda")
    val = torch.empty(M, dtype=torch.float32, device="cuda")
    capi.lm_head_argmax(wt, x.data_ptr(), 896, M, logits.data_ptr(), 0, idx.data_ptr(), val.data_ptr(), stream())
    capi.sync(stream())
    lg = host_u16(logits)
    am = idx.cpu().numpy()
    f = W.f16_bits_to_f32(lg)
    # the device pick is the reference's rule applied to the device logits
    for m in range(M):
        row = f[m]
        best = np.nanmax(row)
        assert am[m] == int(np.flatnonzero(row == best)[0])
        assert val.cpu().numpy()[m] == best
    # and it agrees with the reference's pick wherever the reference's top-2
    # margin exceeds the accumulation noise (one FP16 ulp at that magnitude)
    ref_am = g["argmax"][:M]
    margin = g["margin"][:M]
    ulp = 2.0 ** (np.floor(np.log2(np.abs(f[np.arange(M), am]))) - 10)
    decisive = margin > 2 * ulp
    assert np.all(am[decisive] == ref_am[decisive])
    assert decisive.mean() > 0.9
    truth0 = f64_truth(d["x"][:1], d["w"], FP16)
    check_close(lg[:1], truth0, float(g["ref_err_row0"]), "lm_head row 0", absdot=abs_dot(d["x"][:1], d["w"], FP16),
                K=896)
    np.testing.assert_allclose(f.astype(np.float64).sum(axis=1), g["row_sum"][:M], rtol=1e-3, atol=1.0)


@pytest.fixture(scope="module")
def sweep():
    d = W.sweep_7b()
    g = golden("sweep_7b.npz")
    assert sha(*[d[k] for k in sorted(d)]) == str(g["input_sha"]), "input generator changed"
    return d, g


@pytest.mark.parametrize("name", [n for n, _, _ in W.SWEEP_7B])
def test_sweep_7b(cuda_dev, sweep, name):
    d, g = sweep
    wt = upload(d[name], BF16)
    xfull = d["x_down"] if name == "down" else d["x"]
    xd = dev_u16(xfull)
    rows = g["rows"]
    truths = f64_truth(xfull[rows], d[name], BF16)
    absdots = abs_dot(xfull[rows], d[name], BF16)
    for M in W.SWEEP_M:
        y = gemm(wt, xd[:M])
        sel = rows[rows < M]
        truth = truths[: len(sel)]
        ref = g[f"{name}_rows"][: len(sel)]
        ref_err = rel_frob(ref, truth)
        err = check_close(y[sel], truth, ref_err, f"sweep {name} M={M}", absdot=absdots[: len(sel)],
                          K=xfull.shape[1])
        assert np.mean(y[sel] == ref) > 0.9
        print(f"{name} M={M}: rel err {err:.4e} reference {ref_err:.4e}")
    capi.sync(stream())
