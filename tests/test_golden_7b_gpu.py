"""The 7B-width decoder against the reference's own engine, token for token.

Goldens: tests/golden/decode_7b4l_greedy.json (seed 3) and
decode_7b4l_seed5_greedy.json (seed 5) -- the reference's QwenModel +
InferenceEngine + CpuBackend, built from its sources, greedy-decoding 32
tokens after a 128-token prompt on a seeded random-init checkpoint of the
Qwen2.5-7B width (hidden 3584, 28/4 heads, head_dim 128, intermediate 18944,
vocabulary 152064, RoPE base 1e6, eps 1e-6) with 4 layers
(tests/golden/gen_decode_7b.py --model 7b4l).  The greedy rule is the
reference's first strict maximum (src/engine/inference_engine.cpp:84-95).

The checkpoint (4.1 GB of FP16) is regenerated here from the seed, bit for
bit (its SHA-256 is in the golden), and written once per session as a
safetensors file in a temporary directory.  Three consumers must reproduce
all 32 tokens:

* the device-resident decoder (mrt_decoder_*), per-op step;
* the same decoder with the persistent one-launch step;
* the reference's own QwenModel + InferenceEngine with CudaBackend in
  CpuBackend's place (tests/cpp/_build/ref_engine_cuda), the drop-in.

Every token must be the reference's; the one exception (gpu_util.
check_greedy_tokens) is a step whose reference top-2 logits are a tie at FP16
resolution, where the order of FP32 sums decides and the runner-up is
accepted -- the sequences then part.  Every step's top-2 margin in the
reference's logits is printed, so a failure shows how close the decision was.
"""
from __future__ import annotations

import json
import os
import struct
import sys

import numpy as np
import pytest

from conftest import GOLDEN, ROOT
from gpu_util import check_greedy_tokens
from mruntime_b200 import capi
from mruntime_b200 import workloads as W

sys.path.insert(0, GOLDEN)
import gen_decode_7b as G  # noqa: E402

pytestmark = pytest.mark.gpu

ENGINE_CUDA = os.path.join(ROOT, "tests", "cpp", "_build", "ref_engine_cuda")


GOLDENS = [f for f in ("decode_7b4l_greedy.json", "decode_7b4l_seed5_greedy.json")
           if os.path.exists(os.path.join(GOLDEN, f))]


@pytest.fixture(scope="module", params=GOLDENS)
def ckpt(request, tmp_path_factory):
    with open(os.path.join(GOLDEN, request.param)) as f:
        g = json.load(f)
    d = str(tmp_path_factory.mktemp("decoder_7b4l"))
    paths = G.write_checkpoint(d, g["config"], g["seed"], g["prompt_len"])
    assert paths["weights_sha256"] == g["weights_sha256"], "regenerated weights differ from the golden's"
    assert paths["prompt_sha256"] == g["prompt_sha256"]
    yield g, paths
    for p in ("model", "config", "prompt"):
        os.unlink(paths[p])


def _safetensors_views(path: str):
    """(name, shape, uint16 array mapped from the file) of every tensor."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
    data = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + n)
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        a, b = meta["data_offsets"]
        yield name, tuple(meta["shape"]), data[a:b].view(np.uint16)


def _report(g: dict, toks: list[int], what: str) -> None:
    same = sum(int(a == b) for a, b in zip(toks, g["tokens"]))
    print(f"{what}: {same}/{len(g['tokens'])} tokens equal to the reference engine's")
    print("reference top-2 margins per step: " + " ".join(f"{m:.4f}" for m in g["margins"]))


def _decoder_tokens(g: dict, paths: dict, persistent: bool) -> tuple[list[int], capi.DecoderStats]:
    old = os.environ.get("MRT_DECODE_STEP")
    if persistent:
        os.environ["MRT_DECODE_STEP"] = "persistent"  # read when the decoder finalises, at its first generate
    try:
        dec = capi.Decoder(g["config"], g["prompt_len"] + g["max_new"])
        for name, shape, arr in _safetensors_views(paths["model"]):
            dec.load(name, arr.ctypes.data, capi.FP16, False, shape)
        prompt = W.decoder_prompt(g["seed"], g["prompt_len"], g["config"]["vocab_size"])
        toks, st = dec.generate(prompt, g["max_new"])
        dec.free()
    finally:
        if old is None:
            os.environ.pop("MRT_DECODE_STEP", None)
        else:
            os.environ["MRT_DECODE_STEP"] = old
    return toks, st


def test_decoder_matches_reference_engine_7b_width(cuda_dev, ckpt):
    g, paths = ckpt
    toks, st = _decoder_tokens(g, paths, persistent=False)
    _report(g, toks, "device decoder (per-op step)")
    print(f"prefill {st.prefill_ms:.2f} ms, {st.decode_steps} graph steps in {st.decode_ms:.2f} ms")
    check_greedy_tokens(toks, g, f"device decoder, seed {g['seed']}")


def test_persistent_step_matches_reference_engine_7b_width(cuda_dev, ckpt):
    g, paths = ckpt
    toks, st = _decoder_tokens(g, paths, persistent=True)
    _report(g, toks, "device decoder (persistent step)")
    check_greedy_tokens(toks, g, f"persistent step, seed {g['seed']}")


@pytest.mark.parametrize("profile", [False, True], ids=["plain", "ProfilingBackend"])
def test_reference_engine_on_cuda_backend_7b_width(cuda_dev, ckpt, profile):
    """The reference's QwenModel::forward (qwen_model.cpp:355-377) and
    InferenceEngine::generate (inference_engine.cpp:26-67), unmodified, with
    CudaBackend as their Backend: host tensors, the model's host loops
    between the calls (bias add, KV-cache copy, permutes), every op staged
    through the device."""
    assert os.path.exists(ENGINE_CUDA), f"{ENGINE_CUDA} missing: run `make -C tests/cpp engine_cuda`"
    g, paths = ckpt
    info = G.run_engine(ENGINE_CUDA, paths, g["max_new"], profile=profile, timeout=1200, nice=False)
    _report(g, info["tokens"], info["backend"])
    print(f"generate {info['generate_seconds']:.1f} s")
    same = check_greedy_tokens(info["tokens"], g, f"reference engine on CudaBackend, seed {g['seed']}")
    if same < len(g["tokens"]):
        print(f"CudaBackend logits' own top-2 margin at step {same}: {info['margins'][same]}")
    if profile:
        calls = info["profile"]
        n_forward = g["prompt_len"] + g["max_new"]
        layers = g["config"]["num_hidden_layers"]
        # 7 projections per layer plus lm_head, per forward (qwen_model.cpp:126-128, 256, 278-279, 288, 374)
        assert calls["gemm"]["calls"] == n_forward * (7 * layers + 1)
        assert calls["flash_attention"]["calls"] == n_forward * layers * g["config"]["num_attention_heads"]
