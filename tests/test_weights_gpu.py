"""Safetensors checkpoint ingest into the executor (msgl_model_load_safetensors) on a B200:
a checkpoint in Hugging Face naming, written from the same weights that set_weights takes,
gives bit-identical logits -- with q / k / v and gate / up stored separately or fused, shards
mixing BF16, F16 and F32, and a tied lm_head (absent: the embedding is used). A missing tensor
is reported by name."""
import numpy as np
import pytest
import torch

from test_model_gpu import CFG, weights
from test_safetensors import write_safetensors

pytestmark = pytest.mark.gpu


def hf_tensors(w, cfg, fused, tied):
    """Our tensor names -> the Hugging Face names of Qwen3ForCausalLM."""
    D, hq, hkv, I = cfg["head_dim"], cfg["num_q_heads"], cfg["num_kv_heads"], cfg["inter"]
    out = {"model.embed_tokens.weight": w["embed"], "model.norm.weight": w["norm"]}
    if not tied:
        out["lm_head.weight"] = w["lm_head"]
    for l in range(cfg["num_layers"]):
        p, q = f"model.layers.{l}.", f"layers.{l}."
        out[p + "input_layernorm.weight"] = w[q + "input_ln"]
        out[p + "post_attention_layernorm.weight"] = w[q + "post_ln"]
        out[p + "self_attn.q_norm.weight"] = w[q + "q_norm"]
        out[p + "self_attn.k_norm.weight"] = w[q + "k_norm"]
        out[p + "self_attn.o_proj.weight"] = w[q + "o"]
        out[p + "mlp.down_proj.weight"] = w[q + "down"]
        if fused:
            out[p + "self_attn.qkv_proj.weight"] = w[q + "qkv"]
            out[p + "mlp.gate_up_proj.weight"] = w[q + "gate_up"]
        else:
            qkv = w[q + "qkv"]
            out[p + "self_attn.q_proj.weight"] = qkv[:hq * D]
            out[p + "self_attn.k_proj.weight"] = qkv[hq * D:(hq + hkv) * D]
            out[p + "self_attn.v_proj.weight"] = qkv[(hq + hkv) * D:]
            out[p + "mlp.gate_proj.weight"] = w[q + "gate_up"][:I]
            out[p + "mlp.up_proj.weight"] = w[q + "gate_up"][I:]
    return out


def write_checkpoint(d, tensors):
    """Two shards. The norm gains (bf16 values near 1, exact in F16 and F32) go in as F16
    (the layer norms) and F32 (q / k norms and the final norm), the matrices as BF16, so the
    loader's conversions must reproduce the same bf16 bits."""
    names = sorted(tensors)
    half = len(names) // 2
    for i, chunk in enumerate((names[:half], names[half:])):
        shard = {}
        for n in chunk:
            dt = "F16" if n.endswith("layernorm.weight") else \
                "F32" if n.endswith("norm.weight") else "BF16"
            shard[n] = (tensors[n], dt)
        write_safetensors(d / f"model-0000{i + 1}-of-00002.safetensors", shard, {"format": "pt"})


def run_prefill(model):
    from msgl.model import BatchBuilder, PagePool, Request
    model.alloc_kv(16)
    rng = np.random.default_rng(4)
    reqs = [Request([int(t) for t in rng.integers(0, CFG["vocab"], n)]) for n in (11, 23)]
    sb = BatchBuilder(PagePool(16)).build(reqs, decode=False, max_pages=4)
    nxt, lg = model.forward(sb, logits=True)
    torch.cuda.synchronize()
    return nxt.cpu().numpy(), lg.cpu().numpy()


@pytest.mark.parametrize("fused,tied", [(False, False), (True, True)])
def test_load_safetensors_matches_set_weights(cuda, tmp_path, fused, tied):
    from msgl import ops
    from msgl.model import Qwen3Model
    w = weights(CFG, 8)
    if tied:
        w = dict(w, lm_head=w["embed"])
    write_checkpoint(tmp_path, hf_tensors(w, CFG, fused, tied))
    a = Qwen3Model(CFG, max_tokens=64, max_reqs=4)
    a.load_safetensors(str(tmp_path))
    b = Qwen3Model(CFG, max_tokens=64, max_reqs=4)
    b.set_weights(w)
    ids_a, lg_a = run_prefill(a)
    ids_b, lg_b = run_prefill(b)
    assert np.array_equal(lg_a, lg_b) and np.array_equal(ids_a, ids_b)
    assert ops.device_error() == (0, 0)


def test_load_safetensors_reports_missing_tensor(cuda, tmp_path):
    from msgl import lib
    from msgl.model import Qwen3Model
    w = weights(CFG, 9)
    t = hf_tensors(w, CFG, fused=False, tied=False)
    del t["model.layers.1.self_attn.k_norm.weight"]
    write_checkpoint(tmp_path, t)
    m = Qwen3Model(CFG, max_tokens=64, max_reqs=4)
    with pytest.raises(RuntimeError):
        m.load_safetensors(str(tmp_path))
    assert b"model.layers.1.self_attn.k_norm.weight" in lib().msgl_last_error()
