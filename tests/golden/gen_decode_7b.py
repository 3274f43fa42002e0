"""Golden greedy tokens of the reference's own engine on seeded random-init
Qwen2 decoders (FP16 weights and q/k/v biases ~ N(0, 0.02), RMSNorm gains 1,
RoPE base 1e6, eps 1e-6; prompts uniform in [0, vocab);
mruntime_b200.workloads.decoder_tensors / decoder_prompt).

Models (``--model``):

* ``7b``    the Qwen2.5-7B shape: hidden 3584, 28 layers, 28/4 heads,
            intermediate 18944, vocab 152064; 512-token prompt, 32 tokens,
            seed 3 -> decode_7b_greedy.json (15.2 GB checkpoint; hours of CPU).
* ``7b4l``  the same width with 4 layers; 128-token prompt, 32 tokens, seed 3
            -> decode_7b4l_greedy.json (4.1 GB checkpoint; minutes of CPU).
            Small enough for the GPU suite to regenerate its weights and
            check every token by default.
* ``tiny``  2 layers, 256 wide; 16-token prompt, 8 tokens -> decode_tiny_greedy.json.

Writes the checkpoint as a safetensors file under _data/ (neither committed nor
shipped with the tests: the GPU side regenerates identical bits from the
seed), runs oracle/_ref/ref_engine -- the reference's QwenModel +
InferenceEngine + CpuBackend built from its sources (`make -C oracle engine`)
-- and stores the generated ids, and the top-2 logit margin, best logit and
runner-up id of every pick, beside this script.  A seed other than 3 is
added to the file name (decode_<model>_seed<N>_greedy.json).

    python tests/golden/gen_decode_7b.py [--model tiny|7b4l|7b] [--threads N] [--seed N]
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import struct
import subprocess
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from mruntime_b200 import workloads as W  # noqa: E402

# model tag -> (config, prompt length, new tokens)
MODELS = {
    "tiny": (W.DECODER_TINY, 16, 8),
    "7b4l": (W.DECODER_7B_4L, 128, 32),
    "7b": (W.DECODER_7B, 512, 32),
}


def write_safetensors(path: str, cfg: dict, seed: int) -> str:
    """Write the seeded checkpoint; return the SHA-256 of its tensor bytes."""
    specs = W.decoder_tensor_specs(cfg)
    header, off = {}, 0
    for name, shape, _ in specs:
        n = int(np.prod(shape)) * 2
        header[name] = {"dtype": "F16", "shape": list(shape), "data_offsets": [off, off + n]}
        off += n
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    h = hashlib.sha256()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for name, arr in W.decoder_tensors(seed, cfg):
            b = np.ascontiguousarray(arr).tobytes()
            h.update(b)
            f.write(b)
    return h.hexdigest()


def write_checkpoint(data: str, cfg: dict, seed: int, n_prompt: int) -> dict:
    """Checkpoint, config and prompt files of one golden case under `data`."""
    os.makedirs(data, exist_ok=True)
    paths = {"model": os.path.join(data, "model.safetensors"), "config": os.path.join(data, "config.json"),
             "prompt": os.path.join(data, "prompt.txt")}
    paths["weights_sha256"] = write_safetensors(paths["model"], cfg, seed)
    with open(paths["config"], "w") as f:
        json.dump(cfg, f)
    prompt = W.decoder_prompt(seed, n_prompt, cfg["vocab_size"])
    with open(paths["prompt"], "w") as f:
        f.write(" ".join(str(int(t)) for t in prompt))
    paths["prompt_sha256"] = hashlib.sha256(prompt.tobytes()).hexdigest()
    return paths


def run_engine(binary: str, paths: dict, max_new: int, threads: int = 0, profile: bool = False,
               timeout: float | None = None, nice: bool = True) -> dict:
    """Run a build of oracle/ref_shim/ref_engine.cpp; parse its report."""
    cmd = (["nice", "-n", "19"] if nice else []) + [binary, paths["model"], paths["config"], paths["prompt"],
                                                    str(max_new), str(threads)]
    if profile:
        cmd.append("--profile")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
    if r.returncode != 0:
        raise RuntimeError(f"{os.path.basename(binary)} failed ({r.returncode}):\n{r.stdout[-2000:]}{r.stderr[-2000:]}")
    info: dict = {"profile": {}}
    for line in r.stdout.splitlines():
        key, _, rest = line.partition(" ")
        if key == "TOKENS":
            info["tokens"] = [int(t) for t in rest.split()]
        elif key == "MARGINS":
            info["margins"] = [float(t) for t in rest.split()]
        elif key == "RUNNERS_UP":
            info["runner_up"] = [int(t) for t in rest.split()]
        elif key == "TOP1":
            info["top1"] = [float(t) for t in rest.split()]
        elif key in ("LOAD_SECONDS", "GENERATE_SECONDS", "THREADS"):
            info[key.lower()] = float(rest)
        elif key == "BACKEND":
            info["backend"] = rest
        elif key == "PROFILE":
            op, calls, ns = rest.split()
            info["profile"][op] = {"calls": int(calls), "total_ns": int(ns)}
    return info


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", choices=sorted(MODELS), default="7b")
    ap.add_argument("--threads", type=int, default=0)
    ap.add_argument("--seed", type=int, default=3)
    args = ap.parse_args()
    cfg, n_prompt, max_new = MODELS[args.model]
    tag = args.model if args.seed == 3 else f"{args.model}_seed{args.seed}"
    data = os.path.join(ROOT, "_data", f"decoder_{tag}")
    t0 = time.time()
    paths = write_checkpoint(data, cfg, args.seed, n_prompt)
    print(f"checkpoint written in {time.time() - t0:.0f} s", flush=True)
    info = run_engine(os.path.join(ROOT, "oracle", "_ref", "ref_engine"), paths, max_new, args.threads)
    info.pop("profile", None)
    out = {"config": cfg, "seed": args.seed, "prompt_len": n_prompt, "max_new": max_new,
           "prompt_sha256": paths["prompt_sha256"], "weights_sha256": paths["weights_sha256"],
           "host_cpus": os.cpu_count(), **info}
    dst = os.path.join(HERE, f"decode_{tag}_greedy.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1)
    print(json.dumps({k: v for k, v in out.items() if k != "config"}))


if __name__ == "__main__":
    main()
