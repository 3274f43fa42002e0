"""Safetensors checkpoints straight into device memory (mrt_safetensors_*,
mrt_decoder_load_safetensors) on the GPU: device reads match the file's
bytes, a weight uploaded from the file is the weight uploaded from host
memory (same conversion and tiling), and a decoder loaded from a checkpoint
file picks the reference engine's greedy tokens."""
import json
import os
import struct
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from gpu_util import host_u16, stream
from mruntime_b200 import capi
from mruntime_b200 import workloads as W

sys.path.insert(0, GOLDEN)
import gen_decode_7b as G  # noqa: E402

pytestmark = pytest.mark.gpu


def _weight_rows(wt) -> np.ndarray:
    buf = torch.empty((wt.n, wt.k), dtype=torch.int16, device="cuda")
    wt.read(buf.data_ptr(), stream=stream())
    capi.sync(stream())
    return host_u16(buf)


def test_device_read_and_weight_upload_match_host_path(cuda_dev, tmp_path):
    rng = np.random.default_rng(11)
    w16 = W.to_f16_bits(rng.standard_normal((300, 200), dtype=np.float32) * np.float32(0.02))
    wb = W.to_bf16_bits(rng.standard_normal((257, 136), dtype=np.float32) * np.float32(0.02))
    big = W.to_f16_bits(rng.standard_normal((5000, 1024), dtype=np.float32))  # several 16 MiB staging chunks
    blobs = [("w16", "F16", w16), ("wb", "BF16", wb), ("big", "F16", big)]
    header, off, data = {}, 0, b""
    for name, dt, a in blobs:
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
        data += a.tobytes()
    hb = json.dumps(header).encode()
    p = str(tmp_path / "w.safetensors")
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", len(hb)) + hb + data)
    f = capi.SafeTensors(p)
    # raw bytes into device memory through the pinned staging buffers
    dev = torch.empty(big.size, dtype=torch.int16, device="cuda")
    f.read("big", dev.data_ptr(), big.nbytes, stream())
    np.testing.assert_array_equal(host_u16(dev).reshape(big.shape), big)
    # uploads from the file == uploads from host memory (FP16 as is, BF16 rounded to FP16 once)
    for name, dt, a in blobs[:2]:
        code = capi.FP16 if dt == "F16" else capi.BF16
        from_file = f.upload_weight(name, stream=stream())
        arr = np.ascontiguousarray(a)
        from_host = capi.Weight(arr.ctypes.data, code, False, a.shape[0], a.shape[1], None, None, stream())
        assert (from_file.n, from_file.k) == a.shape
        np.testing.assert_array_equal(_weight_rows(from_file), _weight_rows(from_host))
        from_file.free()
        from_host.free()
    # a shard: rows [8, 40) and [100, 120), columns [64, 128)
    sh = f.upload_weight("w16", row_ranges=[(8, 40), (100, 120)], k_range=(64, 128), stream=stream())
    np.testing.assert_array_equal(_weight_rows(sh), np.concatenate([w16[8:40, 64:128], w16[100:120, 64:128]]))
    sh.free()
    f.close()


def test_decoder_from_checkpoint_matches_reference_engine(cuda_dev, tmp_path):
    with open(os.path.join(GOLDEN, "decode_tiny_greedy.json")) as fh:
        g = json.load(fh)
    paths = G.write_checkpoint(str(tmp_path), g["config"], g["seed"], g["prompt_len"])
    f = capi.SafeTensors(paths["model"])
    dec = capi.Decoder(g["config"], g["prompt_len"] + g["max_new"])
    n = dec.load_safetensors(f)
    assert n == len(W.decoder_tensor_specs(g["config"]))
    prompt = W.decoder_prompt(g["seed"], g["prompt_len"], g["config"]["vocab_size"])
    toks, _ = dec.generate(prompt, g["max_new"])
    assert toks == g["tokens"], f"decoder from checkpoint {toks} != reference {g['tokens']}"
    dec.free()
    f.close()


def test_extra_tensors_are_ignored_like_the_reference(cuda_dev, tmp_path):
    """QwenModel::load_weights reads only the names it knows
    (qwen_model.cpp:336-353); a checkpoint with more tensors loads the same."""
    cfg = W.DECODER_TINY
    tensors = list(W.decoder_tensors(3, cfg))
    extra = [("model.layers.0.self_attn.rotary_emb.inv_freq", np.zeros(32, np.uint16)),
             ("model.layers.7.mlp.up_proj.weight", np.zeros((4, 4), np.uint16)),  # beyond num_layers
             ("lm_head.extra", np.zeros(3, np.uint16))]
    header, off, blobs = {}, 0, []
    for name, a in tensors + extra:
        header[name] = {"dtype": "F16", "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
        blobs.append(np.ascontiguousarray(a).tobytes())
    hb = json.dumps(header).encode()
    p = str(tmp_path / "extra.safetensors")
    with open(p, "wb") as fh:
        fh.write(struct.pack("<Q", len(hb)) + hb + b"".join(blobs))
    f = capi.SafeTensors(p)
    dec = capi.Decoder(cfg, 24)
    assert dec.load_safetensors(f) == len(tensors)
    prompt = W.decoder_prompt(5, 12, cfg["vocab_size"])
    t_file, _ = dec.generate(prompt, 6)
    ref = capi.Decoder(cfg, 24)
    for name, a in tensors:
        arr = np.ascontiguousarray(a)
        ref.load(name, arr.ctypes.data, capi.FP16, False, arr.shape)
    t_host, _ = ref.generate(prompt, 6)
    assert t_file == t_host
    dec.free()
    ref.free()
    f.close()
