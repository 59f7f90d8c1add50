"""Generates the golden fixtures in this folder from the oracle (test infrastructure).

  python tests/golden/make_golden.py

ref_patterns.npz
  The deterministic block patterns of the reference's fused-kernel property
  tests (crates/realm-compute-cpu/src/fused.rs:2840-2915 Q4_K, 3483-3573 Q6_K,
  3648-3726 Q8_0), their input vector, the exact dequantised weights and the
  fused GEMV outputs (computed in double from the exact weights).

tinyllama_c1.npz
  The correctness configuration: TinyLlama-1.1B architecture (22 layers, hidden
  2048, 32 q / 4 kv heads, head_dim 64, FFN 5632, vocab 32000, eps 1e-5, theta
  1e4), random-init N(0, 0.02) weights from seed 0 quantised to Q4_K_M (attn_v
  and output Q6_K), a 40-token prompt U[0, 32000) from seed 1, greedy decode of
  64 tokens with fp32 KV (Model::generate, crates/realm-models/src/model.rs:749-847,
  repetition penalty 1.0). Stored: prompt, the 64 greedy tokens, the full logits
  of steps 0 and 63, and the top-8 (index, logit) of every step.
"""
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))               # tests/ (synth)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))  # repository root (oracle)

from oracle import oracle as O  # noqa: E402
import synth  # noqa: E402

TOP = 8
FULL_STEPS = (0, 63)


def _f16(v):
    return O.f32_to_f16_bits(float(v))


def ref_patterns():
    q4 = b""
    for i in range(2):
        for j in range(2):
            q4 += struct.pack("<HH", _f16(0.5 + i * 0.1), _f16(0.1)) + bytes([16 + i + j] * 12) + \
                bytes([(i * 17 + j * 13) % 256] * 128)
    q6 = b""
    for i in range(2):
        for j in range(2):
            q6 += bytes((i * 15 + j * 9 + t) % 255 for t in range(128)) + \
                bytes((i * 13 + j * 7 + t) % 255 for t in range(64)) + \
                np.array([((i * 9 + j * 5 + t) % 127) - 64 for t in range(16)], np.int8).tobytes() + \
                struct.pack("<H", _f16(0.5 + i * 0.1))
    q8 = b""
    for i in range(2):
        for j in range(2):
            q8 += struct.pack("<H", _f16(0.5 + i * 0.1)) + \
                np.array([((i * 13 + j * 7 + t) % 127) - 64 for t in range(32)], np.int8).tobytes()
    out = {}
    for name, dt, blocks, k in (("q4k", O.Q4K, q4, 512), ("q6k", O.Q6K, q6, 512), ("q80", O.Q80, q8, 64)):
        b = np.frombuffer(blocks, np.uint8)
        x = np.array([((t % 7) - 3.0) * 0.5 for t in range(k)], np.float32)
        w = O.dequant(dt, b).reshape(2, k)
        out[f"{name}_blocks"] = b
        out[f"{name}_x"] = x
        out[f"{name}_w"] = w
        out[f"{name}_y"] = (w.astype(np.float64) @ x.astype(np.float64)).astype(np.float32)
    return out


def tinyllama():
    cfg = synth.TINYLLAMA
    W = synth.make_weights(cfg, seed=0)
    prompt = np.random.default_rng(1).integers(0, cfg["vocab"], 40).astype(np.uint32)
    om = O.Model(dict(cfg, kv_fp16=0), W)
    toks, logits = om.generate(prompt, 64)
    top_idx = np.argsort(-logits, axis=1, kind="stable")[:, :TOP].astype(np.int32)
    top_val = np.take_along_axis(logits, top_idx, axis=1)
    return dict(prompt=prompt, tokens=toks.astype(np.uint32), full_steps=np.array(FULL_STEPS, np.int32),
                full_logits=logits[list(FULL_STEPS)], top_idx=top_idx, top_val=top_val)


def main():
    O.build()
    np.savez_compressed(os.path.join(HERE, "ref_patterns.npz"), **ref_patterns())
    np.savez_compressed(os.path.join(HERE, "tinyllama_c1.npz"), **tinyllama())
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
