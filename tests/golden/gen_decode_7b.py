"""Golden greedy tokens of the reference's own engine on the random-init
Qwen2.5-7B-shaped decoder (hidden 3584, 28 layers, 28/4 heads, intermediate
18944, vocab 152064, FP16 weights and q/k/v biases ~ N(0, 0.02), RMSNorm
gains 1, RoPE base 1e6, eps 1e-6; a 512-token prompt uniform in
[0, 152064); seed 3; mruntime_b200.workloads.decoder_tensors / decoder_prompt).

Writes the checkpoint as a safetensors file under _data/ (15.2 GB; neither
committed nor shipped with the tests: the GPU side regenerates identical bits
from the seed), runs
oracle/_ref/ref_engine -- the reference's QwenModel + InferenceEngine built
from its sources (`make -C oracle engine`) -- and stores the 32 generated ids
in decode_7b_greedy.json beside this script.

    python tests/golden/gen_decode_7b.py [--tiny] [--threads N]

--tiny runs a 2-layer, 256-wide model of the same structure (a pipeline check
that takes seconds; its tokens go to decode_tiny_greedy.json).
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

TINY = W.DECODER_TINY


def write_safetensors(path: str, cfg: dict, seed: int) -> str:
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tiny", action="store_true")
    ap.add_argument("--threads", type=int, default=0)
    ap.add_argument("--seed", type=int, default=3)
    args = ap.parse_args()
    cfg = TINY if args.tiny else W.DECODER_7B
    n_prompt, max_new = (16, 8) if args.tiny else (512, 32)
    tag = "tiny" if args.tiny else "7b"
    data = os.path.join(ROOT, "_data", f"decoder_{tag}")
    os.makedirs(data, exist_ok=True)
    model = os.path.join(data, "model.safetensors")
    t0 = time.time()
    weights_sha = write_safetensors(model, cfg, args.seed)
    with open(os.path.join(data, "config.json"), "w") as f:
        json.dump(cfg, f)
    prompt = W.decoder_prompt(args.seed, n_prompt, cfg["vocab_size"])
    with open(os.path.join(data, "prompt.txt"), "w") as f:
        f.write(" ".join(str(int(t)) for t in prompt))
    print(f"checkpoint written in {time.time() - t0:.0f} s", flush=True)
    engine = os.path.join(ROOT, "oracle", "_ref", "ref_engine")
    cmd = ["nice", "-n", "19", engine, model, os.path.join(data, "config.json"), os.path.join(data, "prompt.txt"),
           str(max_new), str(args.threads)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.exit(r.stderr[-2000:])
    info = {}
    for line in r.stdout.splitlines():
        key, _, rest = line.partition(" ")
        if key == "TOKENS":
            info["tokens"] = [int(t) for t in rest.split()]
        elif key in ("LOAD_SECONDS", "GENERATE_SECONDS", "THREADS"):
            info[key.lower()] = float(rest)
    out = {"config": cfg, "seed": args.seed, "prompt_len": n_prompt, "max_new": max_new,
           "prompt_sha256": hashlib.sha256(prompt.tobytes()).hexdigest(), "weights_sha256": weights_sha,
           "host_cpus": os.cpu_count(), **info}
    dst = os.path.join(HERE, f"decode_{tag}_greedy.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1)
    print(json.dumps({k: v for k, v in out.items() if k != "config"}))


if __name__ == "__main__":
    main()
