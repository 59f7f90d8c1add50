"""Seeded synthetic Q4_K_M-style models for parity tests (test helper).

Weights are N(0, 0.02) fp32 quantised by the oracle's quantiser; norm weights
are 1.0. attn_v and output use Q6_K, everything else Q4_K, as in the configs.
"""
import numpy as np

from oracle import oracle as O

TINYLLAMA = dict(n_layers=22, hidden=2048, n_heads=32, n_kv_heads=4, head_dim=64, ffn=5632, vocab=32000,
                 max_seq=2048, rms_eps=1e-5, layer_eps=1e-5, rope_theta=10000.0)
LLAMA7B = dict(n_layers=32, hidden=4096, n_heads=32, n_kv_heads=32, head_dim=128, ffn=11008, vocab=32000,
               max_seq=4096, rms_eps=1e-5, layer_eps=1e-5, rope_theta=10000.0)
SMALL = dict(n_layers=2, hidden=512, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1536, vocab=1000,
             max_seq=512, rms_eps=1e-5, layer_eps=1e-5, rope_theta=10000.0)


def shapes(cfg):
    H, Q, KV, F, V = (cfg["hidden"], cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"],
                      cfg["ffn"], cfg["vocab"])
    return {O.W_Q: (Q, H), O.W_K: (KV, H), O.W_V: (KV, H), O.W_O: (H, Q), O.W_GATE: (F, H), O.W_UP: (F, H),
            O.W_DOWN: (H, F)}


def make_weights(cfg, seed=0, q_main=O.Q4K, q_v=O.Q6K, q_out=O.Q6K, q_embd=O.Q4K):
    rng = np.random.default_rng(seed)
    H, V = cfg["hidden"], cfg["vocab"]
    W = {}

    def quant(dt, rows, cols):
        x = rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32)
        return dt, O.quantize(dt, x)

    W[(O.W_TOKEN_EMBD, -1)] = quant(q_embd, V, H)
    for l in range(cfg["n_layers"]):
        for which, (r, c) in shapes(cfg).items():
            W[(which, l)] = quant(q_v if which == O.W_V else q_main, r, c)
        W[(O.W_ATTN_NORM, l)] = (O.F32, np.ones(H, np.float32))
        W[(O.W_FFN_NORM, l)] = (O.F32, np.ones(H, np.float32))
    W[(O.W_OUTPUT_NORM, -1)] = (O.F32, np.ones(H, np.float32))
    W[(O.W_OUTPUT, -1)] = quant(q_out, V, H)
    return W
