"""Device-resident greedy decoder against the reference's own engine.

The golden tokens come from the reference's QwenModel + InferenceEngine built
from its sources (oracle/ref_shim/ref_engine.cpp, tests/golden/gen_decode_7b.py)
on seeded random-init checkpoints; the decoder here regenerates the same bits
from the seed and must pick the same greedy tokens.  The full 28-layer
7B-shaped case needs several minutes of host time to regenerate its 15 GB of
weights, so it runs only with MRT_GOLDEN_7B=1; the 7B width with 4 layers
runs by default in test_golden_7b_gpu.py.
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from mruntime_b200 import capi
from mruntime_b200 import workloads as W

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _build(cfg: dict, max_seq: int, seed: int = 3, skip: tuple[str, ...] = ()) -> capi.Decoder:
    dec = capi.Decoder(cfg, max_seq)
    for name, bits in W.decoder_tensors(seed, cfg):
        if name in skip:
            continue
        arr = np.ascontiguousarray(bits)
        dec.load(name, arr.ctypes.data, capi.FP16, False, arr.shape)
    return dec


def _golden(tag: str) -> dict:
    with open(os.path.join(GOLDEN, f"decode_{tag}_greedy.json")) as f:
        return json.load(f)


def test_tiny_matches_reference_engine(cuda_dev):
    g = _golden("tiny")
    cfg = W.DECODER_TINY
    prompt = W.decoder_prompt(g["seed"], g["prompt_len"], cfg["vocab_size"])
    dec = _build(cfg, g["prompt_len"] + g["max_new"], g["seed"])
    toks, st = dec.generate(prompt, g["max_new"])
    assert toks == g["tokens"], f"decoder {toks} != reference {g['tokens']}"
    assert st.decode_steps == g["max_new"] - 2 and st.prefill_ms > 0
    # A second run from the same decoder starts from position 0 again.
    toks2, _ = dec.generate(prompt, g["max_new"])
    assert toks2 == toks
    dec.free()


def test_tiny_eos_stops_after_the_token(cuda_dev):
    g = _golden("tiny")
    cfg = W.DECODER_TINY
    prompt = W.decoder_prompt(g["seed"], g["prompt_len"], cfg["vocab_size"])
    dec = _build(cfg, g["prompt_len"] + g["max_new"], g["seed"])
    eos = g["tokens"][1]
    toks, _ = dec.generate(prompt, g["max_new"], eos=eos)
    assert toks == g["tokens"][: g["tokens"].index(eos) + 1]
    toks1, _ = dec.generate(prompt, 1)
    assert toks1 == g["tokens"][:1]
    dec.free()


def test_tied_lm_head(cuda_dev):
    """Without lm_head.weight the embedding is the output projection
    (qwen_model.cpp:346-352): same as loading the embedding under that name."""
    cfg = W.DECODER_TINY
    prompt = W.decoder_prompt(5, 12, cfg["vocab_size"])
    tied = _build(cfg, 24, 3, skip=("lm_head.weight",))
    t1, _ = tied.generate(prompt, 6)
    explicit = capi.Decoder(cfg, 24)
    emb = None
    for name, bits in W.decoder_tensors(3, cfg):
        if name == "lm_head.weight":
            continue
        arr = np.ascontiguousarray(bits)
        if name == "model.embed_tokens.weight":
            emb = arr
        explicit.load(name, arr.ctypes.data, capi.FP16, False, arr.shape)
    explicit.load("lm_head.weight", emb.ctypes.data, capi.FP16, False, emb.shape)
    t2, _ = explicit.generate(prompt, 6)
    assert t1 == t2
    tied.free()
    explicit.free()


def test_device_and_bf16_sources_load(cuda_dev):
    """Tensors may come from device memory and in BF16 (rounded once to FP16,
    as the reference's converter does for biases)."""
    cfg = W.DECODER_TINY
    prompt = W.decoder_prompt(7, 10, cfg["vocab_size"])
    a = _build(cfg, 16, 3)
    ta, _ = a.generate(prompt, 5)
    b = capi.Decoder(cfg, 16)
    keep = []
    for name, bits in W.decoder_tensors(3, cfg):
        t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda()
        keep.append(t)
        b.load(name, t.data_ptr(), capi.FP16, True, tuple(bits.shape))
    tb, _ = b.generate(prompt, 5)
    assert ta == tb
    a.free()
    b.free()


def test_errors(cuda_dev):
    cfg = W.DECODER_TINY
    dec = capi.Decoder(cfg, 8)
    arr = np.zeros((4,), np.uint16)
    with pytest.raises(capi.MrtError) as e:
        dec.load("model.layers.0.self_attn.qq_proj.weight", arr.ctypes.data, capi.FP16, False, (4,))
    assert e.value.code == 1
    with pytest.raises(capi.MrtError) as e:
        dec.load("model.norm.weight", arr.ctypes.data, capi.FP16, False, (4,))
    assert "expected 256" in str(e.value)
    with pytest.raises(capi.MrtError) as e:
        dec.load("model.layers.9.input_layernorm.weight", arr.ctypes.data, capi.FP16, False, (256,))
    with pytest.raises(capi.MrtError) as e:  # nothing loaded yet
        dec.generate([1, 2, 3], 2)
    assert "embed_tokens" in str(e.value)
    dec.free()
    full = _build(cfg, 8, 3)
    with pytest.raises(capi.MrtError):
        full.generate([1, 2, 3, 4, 5, 6, 7], 4)  # 7 + 4 - 1 > 8 positions
    with pytest.raises(capi.MrtError) as e:
        full.generate([1, 5000], 2)  # outside the vocabulary
    assert "out of range" in str(e.value)
    toks, _ = full.generate([1, 2, 3, 4, 5], 4)  # 5 + 4 - 1 = 8 fits exactly
    assert len(toks) == 4
    full.free()


@pytest.mark.skipif(os.environ.get("MRT_GOLDEN_7B") != "1", reason="set MRT_GOLDEN_7B=1 (regenerates 15 GB of weights)")
def test_7b_matches_reference_engine(cuda_dev):
    path = os.path.join(GOLDEN, "decode_7b_greedy.json")
    if not os.path.exists(path):
        pytest.skip("decode_7b_greedy.json has not been generated")
    g = _golden("7b")
    cfg = W.DECODER_7B
    prompt = W.decoder_prompt(g["seed"], g["prompt_len"], cfg["vocab_size"])
    dec = _build(cfg, g["prompt_len"] + g["max_new"], g["seed"])
    toks, st = dec.generate(prompt, g["max_new"])
    print(f"7B decode: prefill {st.prefill_ms:.1f} ms, {st.decode_steps} steps in {st.decode_ms:.2f} ms "
          f"({1000.0 * st.decode_steps / max(st.decode_ms, 1e-9):.1f} tok/s); tokens {toks}")
    assert toks == g["tokens"], f"decoder {toks} != reference {g['tokens']}"
    dec.free()


class _PersistentStep:
    """Select the persistent decode-step kernel for decoders built inside."""

    def __enter__(self):
        self.old = os.environ.get("MRT_DECODE_STEP")
        os.environ["MRT_DECODE_STEP"] = "persistent"

    def __exit__(self, *exc):
        if self.old is None:
            os.environ.pop("MRT_DECODE_STEP", None)
        else:
            os.environ["MRT_DECODE_STEP"] = self.old


def _dirty_device_memory(mib: int = 64) -> None:
    """Allocate device memory through the library, fill it with non-zero
    values and free it, so buffers a decoder allocates next may start with
    stale contents instead of the driver's zeroed pages."""
    import ctypes as C

    n = (mib << 20) // 2
    ptr = C.c_void_p()
    capi.call("mrt_device_alloc", C.c_size_t(n * 2), C.byref(ptr))
    src = torch.full((n,), 3.0, dtype=torch.float32, device="cuda")
    capi.convert(src.data_ptr(), capi.FP32, ptr.value, capi.FP16, n, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    del src
    capi.call("mrt_device_free", ptr)


@pytest.mark.parametrize("dirty", [False, True])
def test_tiny_persistent_step_matches_reference_engine(cuda_dev, dirty):
    """The persistent step on the tiny model (fewer split-GEMV units than
    CTAs: the tile sums must skip the CTAs that got none), also after stale
    non-zero memory was handed back to the driver."""
    g = _golden("tiny")
    cfg = W.DECODER_TINY
    prompt = W.decoder_prompt(g["seed"], g["prompt_len"], cfg["vocab_size"])
    if dirty:
        _dirty_device_memory()
    with _PersistentStep():  # read when the decoder finalises, at its first generate
        dec = _build(cfg, g["prompt_len"] + g["max_new"], g["seed"])
        toks, st = dec.generate(prompt, g["max_new"])
    assert toks == g["tokens"], f"persistent step {toks} != reference {g['tokens']}"
    assert st.decode_steps == g["max_new"] - 2
    dec.free()
