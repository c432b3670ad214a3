"""Hugging Face safetensors checkpoints: a model saved under HF names (separate q/k/v and
gate/up projections, Mixtral block_sparse_moe experts, Qwen3 q/k norms with tied embeddings) loads back into the engine and
generates the same tokens as the model it was saved from."""
import json
import os

import torch

from lake_b200.engine.llm_engine import LLMEngine


def _deinterleave(gu, inter, half=128):
    t = gu.view(inter // half, 2, half, -1)
    return t[:, 0].reshape(inter, -1), t[:, 1].reshape(inter, -1)


def _hf_state(eng):
    c, w = eng.cfg, eng.model.w
    q, k = c.n_q_heads * c.head_dim, c.n_kv_heads * c.head_dim
    out = {"model.embed_tokens.weight": w["embed_tokens"], "model.norm.weight": w["norm"]}
    if not c.tie_embeddings:
        out["lm_head.weight"] = w["lm_head"]
    for i in range(c.n_layers):
        p, hp = f"layers.{i}.", f"model.layers.{i}."
        qkv = w[p + "qkv_proj"]
        out[hp + "self_attn.q_proj.weight"] = qkv[:q]
        out[hp + "self_attn.k_proj.weight"] = qkv[q:q + k]
        out[hp + "self_attn.v_proj.weight"] = qkv[q + k:]
        out[hp + "self_attn.o_proj.weight"] = w[p + "o_proj"]
        out[hp + "input_layernorm.weight"] = w[p + "input_layernorm"]
        out[hp + "post_attention_layernorm.weight"] = w[p + "post_attention_layernorm"]
        if c.qk_norm:
            out[hp + "self_attn.q_norm.weight"] = w[p + "q_norm"]
            out[hp + "self_attn.k_norm.weight"] = w[p + "k_norm"]
        if c.n_experts:
            out[hp + "block_sparse_moe.gate.weight"] = w[p + "router"]
            gu, dn = w[p + "experts.gate_up_proj"], w[p + "experts.down_proj"]
            for e in range(c.n_experts):
                g, u = _deinterleave(gu[e], c.intermediate)
                out[hp + f"block_sparse_moe.experts.{e}.w1.weight"] = g
                out[hp + f"block_sparse_moe.experts.{e}.w3.weight"] = u
                out[hp + f"block_sparse_moe.experts.{e}.w2.weight"] = dn[e]
        else:
            g, u = _deinterleave(w[p + "gate_up_proj"], c.intermediate)
            out[hp + "mlp.gate_proj.weight"] = g
            out[hp + "mlp.up_proj.weight"] = u
            out[hp + "mlp.down_proj.weight"] = w[p + "down_proj"]
    return {k: v.detach().contiguous().clone() for k, v in out.items()}


def _save(tmp_path, eng, shards=2, **extra):
    from safetensors.torch import save_file

    c = eng.cfg
    arch = {"mixtral": "MixtralForCausalLM", "qwen3": "Qwen3ForCausalLM"}.get(c.arch, "LlamaForCausalLM")
    cfg = {"architectures": [arch],
           "hidden_size": c.hidden, "num_hidden_layers": c.n_layers, "num_attention_heads": c.n_q_heads,
           "num_key_value_heads": c.n_kv_heads, "head_dim": c.head_dim, "intermediate_size": c.intermediate,
           "vocab_size": c.vocab, "rope_theta": c.rope_theta, "rms_norm_eps": c.rms_eps,
           "max_position_embeddings": c.max_position, "tie_word_embeddings": c.tie_embeddings, **extra}
    if c.n_experts:
        cfg.update(num_local_experts=c.n_experts, num_experts_per_tok=c.top_k)
    d = tmp_path / "ckpt"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(cfg))
    state = _hf_state(eng)
    keys = sorted(state)
    wmap = {}
    for s in range(shards):  # shard boundaries split layers' tensors across files
        part = {k: state[k] for k in keys[s::shards]}
        name = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        save_file(part, str(d / name))
        wmap.update({k: name for k in part})
    (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wmap}))
    return str(d)


def test_llama_checkpoint_roundtrip(tmp_path):
    src = LLMEngine("tiny", device="cpu", max_running=4, max_batched_tokens=128, max_model_len=512, num_blocks=64,
                    seed=3)
    path = _save(tmp_path, src)
    prompts = [[(7 * i + j) % 1000 for j in range(30 + 5 * i)] for i in range(3)]
    want = src.generate(prompts, max_new_tokens=6)
    eng = LLMEngine(path, device="cpu", max_running=4, max_batched_tokens=128, max_model_len=512, num_blocks=64)
    assert eng.cfg.hidden == src.cfg.hidden and eng.cfg.n_layers == src.cfg.n_layers
    for k, v in src.model.w.items():
        assert torch.equal(eng.model.w[k].float(), v.float()), k
    assert eng.generate(prompts, max_new_tokens=6) == want


def test_mixtral_checkpoint_roundtrip(tmp_path):
    from lake_b200.models.config import get_config

    cfg = get_config("tiny", n_experts=4, top_k=2, arch="mixtral")
    src = LLMEngine(cfg, device="cpu", max_running=4, max_batched_tokens=128, max_model_len=512, num_blocks=64,
                    seed=5)
    path = _save(tmp_path, src)
    prompts = [[(11 * i + j) % 1000 for j in range(25 + 3 * i)] for i in range(3)]
    want = src.generate(prompts, max_new_tokens=5)
    eng = LLMEngine(path, device="cpu", max_running=4, max_batched_tokens=128, max_model_len=512, num_blocks=64)
    assert eng.cfg.n_experts == 4
    assert eng.generate(prompts, max_new_tokens=5) == want


def test_qwen3_checkpoint_roundtrip_with_tied_embeddings(tmp_path):
    from lake_b200.models.config import get_config

    cfg = get_config("tiny", arch="qwen3", qk_norm=True, tie_embeddings=True)
    src = LLMEngine(cfg, device="cpu", max_running=4, max_batched_tokens=128, max_model_len=512, num_blocks=64,
                    seed=7)
    for i in range(cfg.n_layers):  # non-trivial norm weights so a dropped q/k norm changes the tokens
        for n in ("q_norm", "k_norm"):
            src.model.w[f"layers.{i}.{n}"].uniform_(0.5, 1.5)
    path = _save(tmp_path, src)
    prompts = [[(13 * i + j) % 1000 for j in range(20 + 7 * i)] for i in range(3)]
    want = src.generate(prompts, max_new_tokens=5)
    eng = LLMEngine(path, device="cpu", max_running=4, max_batched_tokens=128, max_model_len=512, num_blocks=64)
    assert eng.cfg.arch == "qwen3" and eng.cfg.qk_norm and eng.cfg.tie_embeddings
    assert eng.model.w["lm_head"].data_ptr() == eng.model.w["embed_tokens"].data_ptr()
    for i in range(cfg.n_layers):
        assert torch.equal(eng.model.w[f"layers.{i}.q_norm"].float(), src.model.w[f"layers.{i}.q_norm"].float())
    assert eng.generate(prompts, max_new_tokens=5) == want


def test_layerwise_sharded_init_equals_sharded_full_model():
    """A tensor-parallel rank generates its weights one tensor at a time and keeps only its
    slice; the slices equal those cut from the whole model built with the same seed."""
    from lake_b200.models.config import get_config
    from lake_b200.models.llama import DecoderLM
    from lake_b200.models.llama_tp import shard_weights

    cfg = get_config("tiny-gpu")
    full = DecoderLM(cfg, "cpu", torch.float32, seed=3)
    for rank in range(2):
        want = shard_weights(full.w, cfg, rank, 2)
        got = DecoderLM(cfg, "cpu", torch.float32, seed=3,
                        shard=lambda n, t, r=rank: shard_weights({n: t}, cfg, r, 2)[n].clone()).w
        assert want.keys() == got.keys()
        for k in want:
            assert torch.equal(want[k], got[k]), k
