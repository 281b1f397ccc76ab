"""Seeded synthetic glm5_next weights for parity tests (test helper).

Distributions follow the reference's synthetic writer (apus
tools/oracle.py:1288-1495): matmul weights N(0, 1/sqrt(K)), norm weights
1 + 0.05 N(0,1), FP8 tensors stored as amax/448 block-scaled E4M3 codes
(tools/oracle.py:307-322), the mHC fn BF16, the router BF16 N(0, 0.05) with an
F32 bias.  Tensor names are the checkpoint names the reference loader
resolves (minus the "model.language_model." prefix).
"""
import math

import numpy as np

import oracle as O


def tiny_config(**over):
    """The shapes of the reference's tiny fixture config (tools/oracle.py:158-
    189): hidden 256, vocab 384, 5 layers (KDA 0,1,2,4; DSA 3; dense 0-2)."""
    kw = dict(hidden_size=256, vocab_size=384, num_hidden_layers=5, rms_norm_eps=1e-5, hc_mult=4,
              hc_sinkhorn_iters=20, hc_eps=1e-6, first_k_dense_replace=3, intermediate_size=256,
              moe_intermediate_size=128, n_routed_experts=8, n_shared_experts=1, num_experts_per_tok=3,
              routed_scaling_factor=2.5, norm_topk_prob=1, swiglu_limit=10.0, num_attention_heads=2,
              q_lora_rank=128, kv_lora_rank=128, qk_nope_head_dim=128, v_head_dim=128, index_n_heads=2,
              index_head_dim=128, index_topk=8, index_kpool=4, index_kpool_always_select_tail=1,
              linear_num_heads=2, linear_head_dim=128, linear_conv_kernel_dim=4, linear_lower_bound=-5.0,
              num_nextn_predict_layers=1)
    kw.update(over)
    L = kw["num_hidden_layers"]
    kw.setdefault("layer_is_dsa", [int(i % 4 == 3) for i in range(L)])
    kw.setdefault("mlp_is_sparse", [int(i >= kw["first_k_dense_replace"]) for i in range(L)])
    return kw


def fp8_store(W):
    """amax/448 F32 scale per 128x128 block, RNE E4M3 codes
    (tools/oracle.py:307-322; the E4M3 rounding is torch's RNE cast, equal to
    c/num.h:110-134 on clamped input)."""
    import torch
    O_, K = W.shape
    nbo, nbk = (O_ + 127) // 128, (K + 127) // 128
    Wp = np.zeros((nbo * 128, nbk * 128), np.float32)
    Wp[:O_, :K] = W
    blocks = Wp.reshape(nbo, 128, nbk, 128).transpose(0, 2, 1, 3)
    amax = np.maximum(np.abs(blocks).max(axis=(2, 3)), np.float32(2.0 ** -126))
    scale = (amax * np.float32(1.0 / 448.0)).astype(np.float32)
    y = np.clip(blocks / scale[:, :, None, None], -448.0, 448.0).astype(np.float32)
    codes = torch.from_numpy(np.ascontiguousarray(y)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    codes = codes.transpose(0, 2, 1, 3).reshape(nbo * 128, nbk * 128)[:O_, :K]
    return np.ascontiguousarray(codes), scale


def gen_weights(kw, seed=1234, has_mtp=True):
    rng = np.random.default_rng(seed)
    d, hc, V = kw["hidden_size"], kw["hc_mult"], kw["vocab_size"]
    W = {}

    def rnd(*shape, std=None):
        return (rng.standard_normal(shape) * (std if std is not None else 1.0 / math.sqrt(shape[-1]))
                ).astype(np.float32)

    def bf16(name, a):
        W[name] = O.bf16_of(a)

    def f32(name, a):
        W[name] = np.ascontiguousarray(a, np.float32)

    def fp8(name, a):
        c, s = fp8_store(a)
        W[name + ".weight"] = c
        W[name + ".weight_scale_inv"] = s

    def norm(name, n):
        bf16(name, (1.0 + 0.05 * rng.standard_normal(n)).astype(np.float32))

    def dsa(L):
        H, ql, kl = kw["num_attention_heads"], kw["q_lora_rank"], kw["kv_lora_rank"]
        qd, vd, IH, ID = kw["qk_nope_head_dim"], kw["v_head_dim"], kw["index_n_heads"], kw["index_head_dim"]
        fp8(f"{L}.self_attn.q_a_proj", rnd(ql, d))
        norm(f"{L}.self_attn.q_a_layernorm.weight", ql)
        fp8(f"{L}.self_attn.q_b_proj", rnd(H * qd, ql))
        fp8(f"{L}.self_attn.kv_a_proj_with_mqa", rnd(kl, d))
        norm(f"{L}.self_attn.kv_a_layernorm.weight", kl)
        bf16(f"{L}.self_attn.kv_b_proj.weight", rnd(H * (qd + vd), kl))
        fp8(f"{L}.self_attn.o_proj", rnd(d, H * vd))
        bf16(f"{L}.self_attn.indexer.wq_b.weight", rnd(IH * ID, ql))
        bf16(f"{L}.self_attn.indexer.wk.weight", rnd(ID, d))
        norm(f"{L}.self_attn.indexer.k_norm.weight", ID)
        bf16(f"{L}.self_attn.indexer.k_norm.bias", (0.05 * rng.standard_normal(ID)).astype(np.float32))
        bf16(f"{L}.self_attn.indexer.weights_proj.weight", rnd(IH, d))
        bf16(f"{L}.self_attn.indexer.index_kpool_compress_ape",
             (0.05 * rng.standard_normal((kw["index_kpool"], ID))).astype(np.float32))
        bf16(f"{L}.self_attn.indexer.index_kpool_compress_gate", rnd(ID, d))

    def moe(L):
        E, inter = kw["n_routed_experts"], kw["moe_intermediate_size"]
        bf16(f"{L}.mlp.gate.weight", (0.05 * rng.standard_normal((E, d))).astype(np.float32))
        f32(f"{L}.mlp.gate.e_score_correction_bias", (0.1 * rng.standard_normal(E)).astype(np.float32))
        for e in range(E):
            fp8(f"{L}.mlp.experts.{e}.gate_proj", rnd(inter, d))
            fp8(f"{L}.mlp.experts.{e}.up_proj", rnd(inter, d))
            fp8(f"{L}.mlp.experts.{e}.down_proj", rnd(d, inter))
        si = inter * kw["n_shared_experts"]
        fp8(f"{L}.mlp.shared_experts.gate_proj", rnd(si, d))
        fp8(f"{L}.mlp.shared_experts.up_proj", rnd(si, d))
        fp8(f"{L}.mlp.shared_experts.down_proj", rnd(d, si))

    nL = kw["num_hidden_layers"]
    for l in range(nL):
        L = f"layers.{l}"
        norm(f"{L}.input_layernorm.weight", d)
        norm(f"{L}.post_attention_layernorm.weight", d)
        if not kw["layer_is_dsa"][l]:
            H, D, K = kw["linear_num_heads"], kw["linear_head_dim"], kw["linear_conv_kernel_dim"]
            qkv = H * D
            for p in "qkv":
                bf16(f"{L}.self_attn.{p}_proj.weight", rnd(qkv, d))
                bf16(f"{L}.self_attn.{p}_conv1d.weight", (0.25 * rng.standard_normal((qkv, K))).astype(np.float32))
            bf16(f"{L}.self_attn.f_a_proj.weight", rnd(D, d))
            bf16(f"{L}.self_attn.f_b_proj.weight", rnd(qkv, D))
            f32(f"{L}.self_attn.A_log", (0.5 * rng.standard_normal(H)).astype(np.float32))
            f32(f"{L}.self_attn.dt_bias", (0.5 * rng.standard_normal(qkv)).astype(np.float32))
            bf16(f"{L}.self_attn.b_proj.weight", rnd(H, d))
            bf16(f"{L}.self_attn.g_a_proj.weight", rnd(D, d))
            bf16(f"{L}.self_attn.g_b_proj.weight", rnd(qkv, D))
            norm(f"{L}.self_attn.o_norm.weight", D)
            bf16(f"{L}.self_attn.o_proj.weight", rnd(d, qkv))
        else:
            dsa(L)
        if not kw["mlp_is_sparse"][l]:
            inter = kw["intermediate_size"]
            fp8(f"{L}.mlp.gate_proj", rnd(inter, d))
            fp8(f"{L}.mlp.up_proj", rnd(inter, d))
            fp8(f"{L}.mlp.down_proj", rnd(d, inter))
        else:
            moe(L)
        mix = (2 + hc) * hc
        for sub in ("attn", "ffn"):
            bf16(f"{L}.hc_{sub}_fn", rnd(mix, hc * d))
            f32(f"{L}.hc_{sub}_base", (0.25 * rng.standard_normal(mix)).astype(np.float32))
            f32(f"{L}.hc_{sub}_scale", (1.0 + 0.1 * rng.standard_normal(3)).astype(np.float32))
    bf16("embed_tokens.weight", rnd(V, d, std=1.0))
    norm("norm.weight", d)
    bf16("lm_head.weight", rnd(V, d))
    if has_mtp:
        L = f"layers.{nL}"
        norm(f"{L}.enorm.weight", d)
        norm(f"{L}.hnorm.weight", d)
        bf16(f"{L}.eh_proj.weight", rnd(d, 2 * d))
        norm(f"{L}.input_layernorm.weight", d)
        norm(f"{L}.post_attention_layernorm.weight", d)
        dsa(L)
        moe(L)
        norm(f"{L}.shared_head.norm.weight", d)
    return W
