"""rb_model_load_gguf on the GPU: a model loaded from a GGUF file of the
synthetic weights decodes with logits bit-identical to the same weights set
tensor by tensor (same bytes reach the same kernels), for the plain layout,
tied output weights (Model::load_from_gguf's fallback, model.rs:373-385: here
the LM head reads token_embd as [vocab][hidden]), f16 norm weights (widened
exactly) and a 64-byte alignment; and the loaded model tracks the oracle's
Model::forward at the north star's logits bound."""
import numpy as np
import pytest

import gguf_writer as GW
import synth

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3


def _decode(m, prompt, steps=5):
    m.tenant_create(0)
    lg, am = m.forward_rows([0] * len(prompt), prompt)
    out = [lg[-1].copy()]
    tok = am[-1]
    for _ in range(steps):
        lg, am = m.forward_rows([0], [tok])
        out.append(lg[-1].copy())
        tok = am[-1]
    return np.stack(out)


def _weights(oracle, f16_norms):
    cfg = synth.SMALL
    W = synth.make_weights(cfg, seed=1)
    if f16_norms:   # norms that f16 holds exactly, so the f16 file and the f32 set_weight agree
        rng = np.random.default_rng(2)
        for key, (dt, data) in list(W.items()):
            if dt == oracle.F32:
                W[key] = (dt, rng.uniform(0.5, 1.5, data.shape).astype(np.float16).astype(np.float32))
    return cfg, W


@pytest.mark.parametrize("variant", ["plain", "tied", "f16_norms", "align64"])
def test_gguf_model_matches_set_weights(ctx, oracle, tmp_path, variant):
    import realm_b200 as rb
    cfg, W = _weights(oracle, variant == "f16_norms")
    blob = GW.model_gguf(cfg, W, tie_output=variant == "tied", f16_norms=variant == "f16_norms",
                         alignment=64 if variant == "align64" else None)
    p = tmp_path / "m.gguf"
    p.write_bytes(blob)
    g = rb.GGUFFile(str(p))
    assert g.model_config()["hidden"] == cfg["hidden"] and g.model_config()["head_dim"] == cfg["head_dim"]
    mg = g.load_model(ctx, kv_dtype=rb.F16, max_tenants=2)
    Wd = dict(W)
    if variant == "tied":
        Wd[(rb.W_OUTPUT, -1)] = W[(rb.W_TOKEN_EMBD, -1)]
    md = rb.Model(ctx, dict(cfg, kv_dtype=rb.F16, max_tenants=2))
    md.set_weights(Wd)
    prompt = np.random.default_rng(3).integers(0, cfg["vocab"], 13).astype(np.uint32)
    a, b = _decode(mg, prompt), _decode(md, prompt)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    if variant == "plain":
        om = oracle.Model(dict(cfg, kv_fp16=1), W)
        ref = om.forward(prompt, 0)
        assert np.all(np.abs(a[0] - ref) <= ATOL + RTOL * np.abs(ref))
    mg.close()
    md.close()
    g.close()


def test_gguf_load_errors(ctx, oracle, tmp_path):
    import realm_b200 as rb
    cfg, W = _weights(oracle, False)
    g = rb.GGUFFile(data=GW.model_gguf(cfg, W))
    with pytest.raises(rb.RealmError) as e:
        g.load_model(ctx, max_tenants=2, ffn=1024)       # shapes disagree with the config
    assert e.value.code == -3 and "blk.0.ffn_gate.weight" in str(e.value)
    blob = GW.model_gguf(cfg, W)                          # rename one tensor: same length, same layout
    g2 = rb.GGUFFile(data=blob.replace(b"blk.1.ffn_down.weight", b"blk.1.ffn_dowX.weight"))
    with pytest.raises(rb.RealmError) as e:
        g2.load_model(ctx, max_tenants=2)
    assert e.value.code == -2 and "blk.1.ffn_down.weight" in str(e.value)
