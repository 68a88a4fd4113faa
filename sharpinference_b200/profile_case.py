"""Runs one hot-path case twice on GPU 0 (for ncu captures of a single
launch with `-s 1 -c 1`): synthetic seeded weights and inputs, device-resident.

  python -m sharpinference_b200.profile_case gemv Q4_K 200064 3072
  python -m sharpinference_b200.profile_case gemv Q8_0 100352 5120
  python -m sharpinference_b200.profile_case batch Q4_K 200064 3072 16
  python -m sharpinference_b200.profile_case gemm Q4_K 200064 3072 512
  python -m sharpinference_b200.profile_case decode mini 64 2
      (Phi-4-mini random-init decoder: 64 prompt steps, then 2 more decode
      steps; each step is one graph of 292 kernel launches)
  python -m sharpinference_b200.profile_case prefill mini 512
      (Phi-4-mini random-init decoder: one batched prefill of 512 prompt
      tokens, one chunk of 512 rows)
  python -m sharpinference_b200.profile_case decode-trace mini 512
      (the persistent decode step: one step at position 512 with its
      per-phase trace, averaged per phase kind over the layers, CTA 0)
"""
from __future__ import annotations

import sys

import numpy as np

from . import native

TYPES = {"Q4_K": native.Q4_K, "Q8_0": native.Q8_0, "F16": native.F16, "F32": native.F32}


def decode(preset: str, prompt_tokens: int, steps: int) -> None:
    from . import phi4
    cfg = dict(phi4.PHI4_MINI if preset == "mini" else phi4.PHI4_14B)
    cfg["context"] = prompt_tokens + steps + 1
    with native.Decoder(cfg) as dec:
        phi4.load_synthetic(dec, cfg, seed=7)
        prompt = phi4.random_prompt(7, prompt_tokens, cfg["vocab"])
        toks = dec.generate(prompt, steps)
        print(f"decode {preset} prompt={prompt_tokens} steps={steps}: last tokens {toks[-3:].tolist()} "
              f"device_error={native.device_error_take(0)}")


def prefill(preset: str, prompt_tokens: int) -> None:
    from . import phi4
    cfg = dict(phi4.PHI4_MINI if preset == "mini" else phi4.PHI4_14B)
    cfg["context"] = prompt_tokens + 1
    with native.Decoder(cfg) as dec:
        phi4.load_synthetic(dec, cfg, seed=7)
        nxt = dec.prefill(phi4.random_prompt(7, prompt_tokens, cfg["vocab"]))
        print(f"prefill {preset} prompt={prompt_tokens}: next token {nxt} device_error={native.device_error_take(0)}")


def decode_trace(preset: str, position: int) -> None:
    import os
    from . import phi4
    os.environ["SI_DECODE_STEP"] = "1"
    os.environ["SI_DECODE_TRACE"] = "1"
    cfg = dict(phi4.PHI4_MINI if preset == "mini" else phi4.PHI4_14B)
    cfg["context"] = position + 2
    with native.Decoder(cfg) as dec:
        phi4.load_synthetic(dec, cfg, seed=7)
        prompt = phi4.random_prompt(7, position + 1, cfg["vocab"])
        dec.generate(prompt[:position], 0)
        dec.generate(prompt[position:], 0)  # the traced step
        t = dec.read("step_trace", dtype=np.uint64).astype(np.int64)
    phases = t.size // 24
    t = t.reshape(3, phases, 8)
    kinds = ["gather"] + ["qkv", "attention", "combine", "out", "gate_up", "down"] * cfg["layers"] + ["lm_head",
                                                                                                   "argmax"]
    rows = {}
    for ph in range(1, phases - 1):
        r = t[0, ph]
        staged = (r[7] - r[0]) / 1e3 if r[7] else 0.0
        rows.setdefault(kinds[ph], []).append(
            [(r[1] - r[0]) / 1e3, (r[0] - t[0, ph - 1, 2]) / 1e3, staged, r[3] / 1e3, r[4] / 1e3, r[5] / 1e3,
             r[6] / 1e3])
    print(f"persistent decode step, {preset}, position {position}: {(t[0, phases - 1, 1] - t[0, 0, 0]) / 1e3:.1f} us")
    print("phase      work  grid-wait  input  | waits: full  pempty  producer-empty  reducer-pfull   (us, CTA 0)")
    for k, v in rows.items():
        a = np.mean(np.array(v), axis=0)
        print(f"{k:9s} " + " ".join(f"{x:7.2f}" for x in a))


def main(argv: list[str]) -> None:
    if argv[0] == "decode":
        decode(argv[1], int(argv[2]), int(argv[3]))
        return
    if argv[0] == "prefill":
        prefill(argv[1], int(argv[2]))
        return
    if argv[0] == "decode-trace":
        decode_trace(argv[1], int(argv[2]))
        return
    kind, tname, n, k = argv[0], argv[1], int(argv[2]), int(argv[3])
    m = int(argv[4]) if len(argv) > 4 else 1
    wt = TYPES[tname]
    blob = native.synth_weights(wt, 4, n, k, 0.02)
    x = native.synth_normal(1004, m * k, 1.0)
    with native.Context(0) as ctx:
        W, X, Y = ctx.buffer(blob.nbytes), ctx.buffer(x.nbytes), ctx.buffer(4 * m * n)
        W.upload(blob), X.upload(x)
        C = ctx.buffer(8)
        C.upload(np.array([0, m], np.int32))
        for _ in range(2):
            if kind == "gemv":
                ctx.matvec(wt, W, X, Y, n, k)
            elif kind == "batch":
                ctx.batch_shared_matvec(wt, W, X, C, Y, m, n, k)
            elif kind == "gemm":
                ctx.matrix_multiply(wt, X, W, Y, m, n, k)
            else:
                raise SystemExit(f"unknown case {kind}")
        ctx.synchronize()
        y = Y.readback().view(np.float32)
        print(f"{kind} {tname} {n}x{k} m={m}: finite={bool(np.all(np.isfinite(y)))} "
              f"device_error={native.device_error_take(0)}")


if __name__ == "__main__":
    main(sys.argv[1:])
