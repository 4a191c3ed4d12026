"""Structural pin of the oracle's Gemma 3 forward: an independent implementation (transformers'
Gemma3ForCausalLM) run on the same dequantized weights must agree within the noise of the reference's
int8 activation quantization, and a deliberately wrong structure (sliding window off by one) must
not. Also checks the oracle against the second restatement in numpy."""
import copy

import numpy as np
import pytest

from gem_b200 import synth
from oracle import numpy_ref
from oracle import oracle as orc


def _hf_model(cfg, path):
    torch = pytest.importorskip("torch")
    tr = pytest.importorskip("transformers")
    import gguf
    from gguf import quants
    r = gguf.GGUFReader(str(path))
    T = {t.name: t for t in r.tensors}

    def deq(name):
        t = T[name]
        a = np.asarray(quants.dequantize(t.data, t.tensor_type), np.float32)
        if len(t.shape) == 2:
            a = a.reshape(int(t.shape[1]), int(t.shape[0]))
        return torch.tensor(a.reshape(-1) if len(t.shape) == 1 else a)

    c = tr.Gemma3TextConfig(
        vocab_size=cfg["vocab"], hidden_size=cfg["d"], intermediate_size=cfg["ff"], num_hidden_layers=cfg["layers"],
        num_attention_heads=cfg["nh"], num_key_value_heads=cfg["nkv"], head_dim=cfg["hd"], rms_norm_eps=cfg["eps"],
        sliding_window=cfg["window"], query_pre_attn_scalar=cfg["hd"], max_position_embeddings=4096,
        layer_types=["sliding_attention" if l % 6 < 5 else "full_attention" for l in range(cfg["layers"])],
        rope_parameters={"sliding_attention": {"rope_type": "default", "rope_theta": 10000.0},
                         "full_attention": {"rope_type": "default", "rope_theta": cfg["rope_base"]}},
        tie_word_embeddings=True, attn_implementation="eager")
    sd = {"model.embed_tokens.weight": deq("token_embd.weight"), "model.norm.weight": deq("output_norm.weight") - 1}
    names = {"attn_q.weight": "self_attn.q_proj.weight", "attn_k.weight": "self_attn.k_proj.weight",
             "attn_v.weight": "self_attn.v_proj.weight", "attn_output.weight": "self_attn.o_proj.weight",
             "ffn_gate.weight": "mlp.gate_proj.weight", "ffn_up.weight": "mlp.up_proj.weight",
             "ffn_down.weight": "mlp.down_proj.weight"}
    norms = {"attn_norm.weight": "input_layernorm.weight", "attn_q_norm.weight": "self_attn.q_norm.weight",
             "attn_k_norm.weight": "self_attn.k_norm.weight", "post_attention_norm.weight": "post_attention_layernorm.weight",
             "ffn_norm.weight": "pre_feedforward_layernorm.weight", "post_ffw_norm.weight": "post_feedforward_layernorm.weight"}
    for l in range(cfg["layers"]):
        for a, b in names.items():
            sd[f"model.layers.{l}.{b}"] = deq(f"blk.{l}.{a}")
        for a, b in norms.items():  # GGUF folds Gemma's (1 + w) into the stored weight
            sd[f"model.layers.{l}.{b}"] = deq(f"blk.{l}.{a}") - 1

    def build(conf):
        m = tr.Gemma3ForCausalLM(conf).float().eval()
        m.load_state_dict(sd, strict=False)
        return m
    return c, build


def _hf_logprobs(m, toks, n):
    import torch
    with torch.no_grad():
        lg = m(torch.tensor(toks[None, :n].astype(np.int64))).logits[0].double()
    return torch.log_softmax(lg, -1)[torch.arange(n), torch.tensor(toks[1:n + 1].astype(np.int64))].numpy()


def test_oracle_forward_matches_transformers_gemma3(small, threads):
    cfg = small.cfg
    c, build = _hf_model(cfg, small.gguf)
    n = 40
    toks = synth.tokens(n + 1, cfg["vocab"])
    o = orc.Model(small.gguf, ctx=128, threads=threads)
    lp, _, _, _ = o.score(toks, 0)
    d = np.abs(lp - _hf_logprobs(build(c), toks, n))
    assert d.max() < 0.05 and d.mean() < 0.015, (d.max(), d.mean())
    bad = copy.deepcopy(c)
    bad.sliding_window = cfg["window"] + 1
    d_bad = np.abs(lp - _hf_logprobs(build(bad), toks, n))
    assert d_bad.max() > 0.2, d_bad.max()


def test_oracle_matches_numpy_restatement(small):
    o = orc.Model(small.gguf, ctx=64, threads=1)
    nref = numpy_ref.Model(small.gguf, ctx=64)
    toks = synth.tokens(20, small.cfg["vocab"], seed=8)
    worst = 0.0
    for i, t in enumerate(toks):
        hn, ho = nref.forward(int(t), i), o.forward(int(t), i)
        worst = max(worst, float(np.abs(hn - ho).mean()))
    # float64 reductions in numpy vs sequential float32 in the oracle: ~1e-7 until an int8 code flips;
    # a flip is bounded by the quantization noise (one int8 step of one block, the same size as the
    # spread between the reference's own AVX-512 and AVX2 paths, which sum in different orders)
    assert worst < 2e-2


@pytest.fixture(scope="module")
def small_qwen2(model_dir):
    return synth.ensure("small-qwen2", classes=64, directory=model_dir)


def qwen2_logprobs(files, toks):
    """transformers' Qwen2ForCausalLM on the dequantized weights of a synthetic qwen2 GGUF: the log-prob
    of toks[i + 1] after toks[:i + 1] for every i < len(toks) - 1."""
    torch = pytest.importorskip("torch")
    tr = pytest.importorskip("transformers")
    import gguf
    from gguf import quants
    cfg = files.cfg
    r = gguf.GGUFReader(str(files.gguf))
    T = {t.name: t for t in r.tensors}

    def deq(name):
        t = T[name]
        a = np.asarray(quants.dequantize(t.data, t.tensor_type), np.float32)
        if len(t.shape) == 2:
            a = a.reshape(int(t.shape[1]), int(t.shape[0]))
        return torch.tensor(a.reshape(-1) if len(t.shape) == 1 else a)

    c = tr.Qwen2Config(vocab_size=cfg["vocab"], hidden_size=cfg["d"], intermediate_size=cfg["ff"],
                       num_hidden_layers=cfg["layers"], num_attention_heads=cfg["nh"], num_key_value_heads=cfg["nkv"],
                       head_dim=cfg["hd"], rms_norm_eps=cfg["eps"], rope_theta=cfg["rope_base"],
                       max_position_embeddings=4096, tie_word_embeddings=False, attn_implementation="eager")
    sd = {"model.embed_tokens.weight": deq("token_embd.weight"), "lm_head.weight": deq("output.weight"),
          "model.norm.weight": deq("output_norm.weight")}
    names = {"attn_q.weight": "self_attn.q_proj.weight", "attn_k.weight": "self_attn.k_proj.weight",
             "attn_v.weight": "self_attn.v_proj.weight", "attn_q.bias": "self_attn.q_proj.bias",
             "attn_k.bias": "self_attn.k_proj.bias", "attn_v.bias": "self_attn.v_proj.bias",
             "attn_output.weight": "self_attn.o_proj.weight", "ffn_gate.weight": "mlp.gate_proj.weight",
             "ffn_up.weight": "mlp.up_proj.weight", "ffn_down.weight": "mlp.down_proj.weight",
             "attn_norm.weight": "input_layernorm.weight", "ffn_norm.weight": "post_attention_layernorm.weight"}
    for l in range(cfg["layers"]):
        for a, b in names.items():
            sd[f"model.layers.{l}.{b}"] = deq(f"blk.{l}.{a}")
    m = tr.Qwen2ForCausalLM(c).float().eval()
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected and all("rotary" in k for k in missing), (missing, unexpected)
    n = len(toks) - 1
    with torch.no_grad():
        lg = m(torch.tensor(toks[None, :n].astype(np.int64))).logits[0].double()
    return torch.log_softmax(lg, -1)[torch.arange(n), torch.tensor(toks[1:n + 1].astype(np.int64))].numpy()


def test_oracle_qwen2_forward_matches_transformers(small_qwen2, threads):
    """The qwen2 branch (model.rs:160-161, 188-190, 311-315, 400-407: q/k/v biases, SiLU, untied output,
    no embedding scale, every layer global) against transformers' Qwen2 on the same weights."""
    toks = synth.tokens(41, small_qwen2.cfg["vocab"], seed=9)
    o = orc.Model(small_qwen2.gguf, ctx=128, threads=threads)
    lp, _, _, _ = o.score(toks, 0)
    d = np.abs(lp - qwen2_logprobs(small_qwen2, toks))
    assert d.max() < 0.05 and d.mean() < 0.015, (d.max(), d.mean())
