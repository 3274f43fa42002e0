"""Seeded synthetic inputs for the linear-layer workloads.

No public dataset is involved: every input is drawn from numpy's PCG64
generator (``default_rng(seed)``) in float32 and rounded with the reference's
own rules -- FP16 by round-to-nearest-even (numpy's float16 cast is the same
rule as float_to_fp16_bits, reference include/mruntime/dtype.h:39-119, for
every non-NaN input) and BF16 by the reference's add-0x7FFF-plus-lsb trick
(dtype.h:153-160).  16-bit arrays are returned as uint16 bit patterns.

Workloads (sizes are the Qwen2.5 shapes):

* ``decode_gemv``       x[1,896] ~ N(0,1) FP16, W[4864,896] ~ N(0,0.02) FP16, seed 0
                        (one gate_proj GEMV of Qwen2.5-0.5B).
* ``layer_prefill_05b`` one Qwen2.5-0.5B layer's projections at M=512, seed 1:
                        x[512,896] ~ N(0,1) FP16; BF16 weights ~ N(0,0.02) q 896x896,
                        k 128x896, v 128x896, o 896x896, gate 4864x896, up 4864x896,
                        down 896x4864; BF16 biases on q/k/v ~ N(0,0.02); the down
                        projection reads its own x_down[512,4864] ~ N(0,1) FP16.
* ``lm_head_05b``       tied lm_head W[151936,896] ~ N(0,0.02) FP16, x[128,896] ~ N(0,1)
                        FP16 (M=1 uses row 0), seed 2.
* ``sweep_7b``          Qwen2.5-7B projection sweep, seed 4: BF16 weights ~ N(0,0.02)
                        qkv 4608x3584 (q 3584 + k 512 + v 512 rows), o 3584x3584,
                        gate+up 37888x3584 (gate 18944 + up 18944 rows), down 3584x18944;
                        x[2048,3584] and x_down[2048,18944] ~ N(0,1) FP16, M in
                        {1,4,16,64,128,512,2048} uses the first M rows.
"""
from __future__ import annotations

import numpy as np

SWEEP_M = (1, 4, 16, 64, 128, 512, 2048)


def to_f16_bits(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)


def f16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(h, dtype=np.uint16).view(np.float16).astype(np.float32)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def bf16_to_f16_bits(b: np.ndarray) -> np.ndarray:
    """The reference's BF16 -> FP16 packing conversion (cpu_backend.cpp:48-55)."""
    return to_f16_bits(bf16_bits_to_f32(b))


def _normal(rng: np.random.Generator, shape, std: float = 1.0) -> np.ndarray:
    x = rng.standard_normal(shape, dtype=np.float32)
    if std != 1.0:
        x *= np.float32(std)
    return x


def decode_gemv(seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    x = to_f16_bits(_normal(rng, (1, 896)))
    w = to_f16_bits(_normal(rng, (4864, 896), 0.02))
    return {"x": x, "w": w, "w_dtype": 0}


LAYER_05B = (("q", 896, 896), ("k", 128, 896), ("v", 128, 896), ("o", 896, 896),
             ("gate", 4864, 896), ("up", 4864, 896), ("down", 896, 4864))


def layer_prefill_05b(seed: int = 1, M: int = 512) -> dict:
    rng = np.random.default_rng(seed)
    out = {"x": to_f16_bits(_normal(rng, (512, 896)))[:M]}
    for name, n, k in LAYER_05B:
        out[name] = to_bf16_bits(_normal(rng, (n, k), 0.02))
    for name, n in (("bq", 896), ("bk", 128), ("bv", 128)):
        out[name] = to_bf16_bits(_normal(rng, (n,), 0.02))
    out["x_down"] = to_f16_bits(_normal(rng, (512, 4864)))[:M]
    return out


def lm_head_05b(seed: int = 2) -> dict:
    rng = np.random.default_rng(seed)
    w = to_f16_bits(_normal(rng, (151936, 896), 0.02))
    x = to_f16_bits(_normal(rng, (128, 896)))
    return {"w": w, "x": x}


SWEEP_7B = (("qkv", (3584, 512, 512), 3584), ("o", (3584,), 3584), ("gateup", (18944, 18944), 3584),
            ("down", (3584,), 18944))
# Column-parallel (split rows) or row-parallel (split K) under tensor parallelism.
SWEEP_7B_PARALLEL = {"qkv": "col", "o": "row", "gateup": "col", "down": "row"}


def sweep_7b(seed: int = 4, max_m: int = 2048) -> dict:
    rng = np.random.default_rng(seed)
    out = {}
    for name, parts, k in SWEEP_7B:
        out[name] = to_bf16_bits(_normal(rng, (sum(parts), k), 0.02))
    out["x"] = to_f16_bits(_normal(rng, (2048, 3584)))[:max_m]
    out["x_down"] = to_f16_bits(_normal(rng, (2048, 18944)))[:max_m]
    return out


DECODER_7B = {
    "vocab_size": 152064, "hidden_size": 3584, "num_hidden_layers": 28, "num_attention_heads": 28,
    "num_key_value_heads": 4, "intermediate_size": 18944, "rope_theta": 1000000.0, "rms_norm_eps": 1e-6,
    "max_position_embeddings": 32768,
}


# The 7B width (hidden 3584, 28/4 heads, intermediate 18944, vocabulary 152064)
# with 4 layers: every projection and the lm_head at full 7B size, small
# enough that the reference engine regenerates its golden tokens in minutes.
DECODER_7B_4L = dict(DECODER_7B, num_hidden_layers=4)


# A 2-layer, 256-wide model of the same structure (head_dim 64, 2 kv heads):
# the quick pipeline check of the decoder against the reference engine.
DECODER_TINY = {
    "vocab_size": 1000, "hidden_size": 256, "num_hidden_layers": 2, "num_attention_heads": 4,
    "num_key_value_heads": 2, "intermediate_size": 512, "rope_theta": 1000000.0, "rms_norm_eps": 1e-6,
    "max_position_embeddings": 32768,
}


def decoder_prompt(seed: int = 3, n: int = 512, vocab: int = 152064) -> np.ndarray:
    """Prompt token ids, uniform in [0, vocab), from the first child stream of `seed`."""
    prompt_ss, _ = np.random.SeedSequence(seed).spawn(2)
    return np.random.default_rng(prompt_ss).integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)


def decoder_tensor_specs(cfg: dict = DECODER_7B):
    """(name, shape, kind) of every tensor of a Qwen2 checkpoint in the
    reference's naming (src/models/qwen/qwen_model.cpp:54-101, 336-353), in
    generation order; kind is "normal" (N(0, 0.02)) or "ones" (RMSNorm gains)."""
    h, inter, v = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    hd = h // cfg["num_attention_heads"]
    kv = cfg["num_key_value_heads"] * hd
    specs = [("model.embed_tokens.weight", (v, h), "normal")]
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}"
        specs += [(f"{p}.input_layernorm.weight", (h,), "ones"),
                  (f"{p}.self_attn.q_proj.weight", (h, h), "normal"), (f"{p}.self_attn.q_proj.bias", (h,), "normal"),
                  (f"{p}.self_attn.k_proj.weight", (kv, h), "normal"), (f"{p}.self_attn.k_proj.bias", (kv,), "normal"),
                  (f"{p}.self_attn.v_proj.weight", (kv, h), "normal"), (f"{p}.self_attn.v_proj.bias", (kv,), "normal"),
                  (f"{p}.self_attn.o_proj.weight", (h, h), "normal"),
                  (f"{p}.post_attention_layernorm.weight", (h,), "ones"),
                  (f"{p}.mlp.gate_proj.weight", (inter, h), "normal"), (f"{p}.mlp.up_proj.weight", (inter, h), "normal"),
                  (f"{p}.mlp.down_proj.weight", (h, inter), "normal")]
    specs += [("model.norm.weight", (h,), "ones"), ("lm_head.weight", (v, h), "normal")]
    return specs


def decoder_tensors(seed: int = 3, cfg: dict = DECODER_7B):
    """Yield (name, FP16 bits) of a random-init Qwen2 decoder: every weight and
    the q/k/v biases ~ N(0, 0.02), RMSNorm gains = 1, from the second child
    stream of `seed`, in decoder_tensor_specs order."""
    _, weight_ss = np.random.SeedSequence(seed).spawn(2)
    rng = np.random.default_rng(weight_ss)
    one = np.uint16(0x3C00)
    for name, shape, kind in decoder_tensor_specs(cfg):
        if kind == "ones":
            yield name, np.full(shape, one, dtype=np.uint16)
        else:
            yield name, to_f16_bits(_normal(rng, shape, 0.02))


def sweep_flops(M: int) -> float:
    return float(sum(2.0 * M * sum(parts) * k for _, parts, k in SWEEP_7B))


def sweep_bytes(M: int) -> float:
    """Algorithmic bytes of one sweep step: FP16 weights + x + y."""
    return float(sum(2.0 * (sum(parts) * k + M * k + M * sum(parts)) for _, parts, k in SWEEP_7B))
