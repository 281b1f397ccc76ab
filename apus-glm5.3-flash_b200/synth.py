"""synth.py — the tensor inventory of a glm5_next model and seeded synthetic
weights for it (pure Python; loads no CUDA library, so the reference arm of
the bench and CPU-only tests can use it).

  tensor_specs(kw)  every checkpoint tensor the engine's set() accepts, with
                    shape, dtype and kind (c/gmodel.h:622-1106 names minus
                    the "model.language_model." prefix)
  ep_owns(kw, r, w) the expert-parallel split of those tensors
  c2_config()       BASELINE config 2 (the scaled 4-layer stack)
  c3_config()       BASELINE config 3 (the full-depth model, real dims)
  c2_weights(...)   seeded weights with BASELINE's distributions
"""


def ep_owns(kw, rank, world):
    """Predicate over checkpoint names: does expert-parallel `rank` of `world`
    store this tensor?  Routed expert e lives on rank e // (E / world); every
    other tensor is stored on every rank (the lm_head as a row slice).  This
    is the split apus_gcuda_model_set applies."""
    E = kw["n_routed_experts"]
    if world > 1 and E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    per = E // world if world > 1 else E

    def owns(name):
        i = name.find(".mlp.experts.")
        if world == 1 or i < 0:
            return True
        e = int(name[i + len(".mlp.experts."):].split(".", 1)[0])
        return e // per == rank
    return owns


def tensor_specs(kw, has_mtp=True):
    """Every tensor GModel.set accepts for config kw: (checkpoint name, shape,
    numpy dtype, kind).  kind: 'bf16' (uint16 codes), 'f32', 'e4m3' (uint8
    codes) or 'scale' (F32 128x128 block scales of the preceding e4m3)."""
    d, V, hc, L = kw["hidden_size"], kw["vocab_size"], kw["hc_mult"], kw["num_hidden_layers"]
    H, D, K = kw["linear_num_heads"], kw["linear_head_dim"], kw["linear_conv_kernel_dim"]
    qkv, mix = H * D, (2 + hc) * hc
    AH, qd, vd = kw["num_attention_heads"], kw["qk_nope_head_dim"], kw["v_head_dim"]
    ql, kl, IH, ID = kw["q_lora_rank"], kw["kv_lora_rank"], kw["index_n_heads"], kw["index_head_dim"]
    E, inter, dense = kw["n_routed_experts"], kw["moe_intermediate_size"], kw["intermediate_size"]
    cb = lambda n: (n + 127) // 128
    out = []

    def t(name, shape, kind):
        dt = {"bf16": "uint16", "f32": "float32", "e4m3": "uint8", "scale": "float32"}[kind]
        out.append((name, tuple(shape), dt, kind))

    def fp8(name, O_, K_):
        t(name + ".weight", (O_, K_), "e4m3")
        t(name + ".weight_scale_inv", (cb(O_), cb(K_)), "scale")

    def dsa(p):
        fp8(p + "self_attn.q_a_proj", ql, d)
        t(p + "self_attn.q_a_layernorm.weight", (ql,), "bf16")
        fp8(p + "self_attn.q_b_proj", AH * qd, ql)
        fp8(p + "self_attn.kv_a_proj_with_mqa", kl, d)
        t(p + "self_attn.kv_a_layernorm.weight", (kl,), "bf16")
        t(p + "self_attn.kv_b_proj.weight", (AH * (qd + vd), kl), "bf16")
        fp8(p + "self_attn.o_proj", d, AH * vd)
        t(p + "self_attn.indexer.wq_b.weight", (IH * ID, ql), "bf16")
        t(p + "self_attn.indexer.wk.weight", (ID, d), "bf16")
        t(p + "self_attn.indexer.k_norm.weight", (ID,), "bf16")
        t(p + "self_attn.indexer.k_norm.bias", (ID,), "bf16")
        t(p + "self_attn.indexer.weights_proj.weight", (IH, d), "bf16")
        t(p + "self_attn.indexer.index_kpool_compress_ape", (kw["index_kpool"], ID), "bf16")
        t(p + "self_attn.indexer.index_kpool_compress_gate", (ID, d), "bf16")

    def moe(p):
        t(p + "mlp.gate.weight", (E, d), "bf16")
        t(p + "mlp.gate.e_score_correction_bias", (E,), "f32")
        for e in range(E):
            fp8(f"{p}mlp.experts.{e}.gate_proj", inter, d)
            fp8(f"{p}mlp.experts.{e}.up_proj", inter, d)
            fp8(f"{p}mlp.experts.{e}.down_proj", d, inter)
        fp8(p + "mlp.shared_experts.gate_proj", inter, d)
        fp8(p + "mlp.shared_experts.up_proj", inter, d)
        fp8(p + "mlp.shared_experts.down_proj", d, inter)

    t("embed_tokens.weight", (V, d), "bf16")
    t("norm.weight", (d,), "bf16")
    t("lm_head.weight", (V, d), "bf16")
    for l in range(L):
        p = f"layers.{l}."
        t(p + "input_layernorm.weight", (d,), "bf16")
        t(p + "post_attention_layernorm.weight", (d,), "bf16")
        for site in ("attn", "ffn"):
            t(p + f"hc_{site}_fn", (mix, hc * d), "bf16")
            t(p + f"hc_{site}_base", (mix,), "f32")
            t(p + f"hc_{site}_scale", (3,), "f32")
        if not kw["layer_is_dsa"][l]:
            for n in "qkv":
                t(p + f"self_attn.{n}_proj.weight", (qkv, d), "bf16")
                t(p + f"self_attn.{n}_conv1d.weight", (qkv, K), "bf16")
            t(p + "self_attn.f_a_proj.weight", (D, d), "bf16")
            t(p + "self_attn.f_b_proj.weight", (qkv, D), "bf16")
            t(p + "self_attn.g_a_proj.weight", (D, d), "bf16")
            t(p + "self_attn.g_b_proj.weight", (qkv, D), "bf16")
            t(p + "self_attn.b_proj.weight", (H, d), "bf16")
            t(p + "self_attn.A_log", (H,), "f32")
            t(p + "self_attn.dt_bias", (qkv,), "f32")
            t(p + "self_attn.o_norm.weight", (D,), "bf16")
            t(p + "self_attn.o_proj.weight", (d, qkv), "bf16")
        else:
            dsa(p)
        if kw["mlp_is_sparse"][l]:
            moe(p)
        else:
            fp8(p + "mlp.gate_proj", dense, d)
            fp8(p + "mlp.up_proj", dense, d)
            fp8(p + "mlp.down_proj", d, dense)
    if has_mtp:
        p = f"layers.{L}."
        t(p + "enorm.weight", (d,), "bf16")
        t(p + "hnorm.weight", (d,), "bf16")
        t(p + "eh_proj.weight", (d, 2 * d), "bf16")
        t(p + "input_layernorm.weight", (d,), "bf16")
        t(p + "post_attention_layernorm.weight", (d,), "bf16")
        dsa(p)
        moe(p)
        t(p + "shared_head.norm.weight", (d,), "bf16")
    return out


def c2_config(small=False):
    """4 layers at hidden 4096 (3 KDA 32x128 + DSA at layer
    3 with the real MLA / Lightning-indexer dims), every layer the config-1
    MoE (288 experts top-8 + shared, inter 1024), vocab 154880, one NextN
    layer.  Other fields from the reference's config.json."""
    kw = dict(hidden_size=4096, vocab_size=154880, num_hidden_layers=4, rms_norm_eps=1e-5, hc_mult=4,
              hc_sinkhorn_iters=20, hc_eps=1e-6, first_k_dense_replace=0, intermediate_size=12288,
              moe_intermediate_size=1024, n_routed_experts=288, n_shared_experts=1, num_experts_per_tok=8,
              routed_scaling_factor=2.5, norm_topk_prob=1, swiglu_limit=10.0, num_attention_heads=64,
              q_lora_rank=1536, kv_lora_rank=512, qk_nope_head_dim=256, v_head_dim=256, index_n_heads=32,
              index_head_dim=128, index_topk=2048, index_kpool=4, index_kpool_always_select_tail=1,
              linear_num_heads=32, linear_head_dim=128, linear_conv_kernel_dim=4, linear_lower_bound=-5.0,
              num_nextn_predict_layers=1, layer_is_dsa=[0, 0, 0, 1], mlp_is_sparse=[1, 1, 1, 1])
    if small:
        kw.update(n_routed_experts=16, vocab_size=16384)
    return kw


def c3_config(layers=45):
    """the full-depth glm5_next at the reference's real
    dims (reference/config.json): 45 layers, DSA at every 4th (i % 4 == 3,
    11 of them) and KDA elsewhere (34, 64 heads x 128), dense MLPs in the
    first 3 layers (intermediate 12288), then MoE of 288 experts top-8 plus
    the shared expert at inter 2048; vocab 154880; one NextN layer.
    `layers` < 45 keeps the same per-layer dims over fewer layers (tests)."""
    L = layers
    kw = dict(c2_config(), num_hidden_layers=L, first_k_dense_replace=3, moe_intermediate_size=2048,
              linear_num_heads=64)
    kw["layer_is_dsa"] = [int(i % 4 == 3) for i in range(L)]
    kw["mlp_is_sparse"] = [int(i >= 3) for i in range(L)]
    return kw


def c2_weights(kw, seed, keep=None):
    """Seeded synthetic weights for every tensor of tensor_specs(kw), made
    with torch on the GPU and returned as host numpy arrays (both bench arms
    load the same arrays).  Experts: BASELINE config 0 codes (E4M3 of
    N(0,1)*64) with log-uniform [1e-4, 1e-2] block scales; router BF16
    N(0, 0.02) with a zero bias; embeddings and head BF16 N(0, 0.02); the DSA
    FP8 linears amax/448 block-scaled N(0, 1/sqrt(K)); BF16 matrices
    N(0, 1/sqrt(K)); norms 1 + 0.05 N(0,1).  keep(name): tensors to return
    (the others are still drawn, so every rank sees the same stream)."""
    import math
    import numpy as np
    import torch
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    g = torch.Generator(device=dev).manual_seed(seed)
    out = {}
    specs = tensor_specs(kw)
    expert = lambda n: ".mlp." in n

    def bf16(t):
        return t.to(torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16)

    i = 0
    while i < len(specs):
        name, shape, dt, kind = specs[i]
        if kind == "e4m3":
            sname, sshape = specs[i + 1][0], specs[i + 1][1]
            O_, K_ = shape
            if expert(name):
                v = torch.clamp(torch.randn(shape, generator=g, device=dev) * 64, -448, 448)
                codes = v.to(torch.float8_e4m3fn)
                lo, hi = math.log(1e-4), math.log(1e-2)
                sc = torch.exp(lo + (hi - lo) * torch.rand(sshape, generator=g, device=dev))
            else:
                w = torch.randn(shape, generator=g, device=dev) / math.sqrt(K_)
                nbo, nbk = sshape
                wp = torch.zeros((nbo * 128, nbk * 128), device=dev)
                wp[:O_, :K_] = w
                blk = wp.view(nbo, 128, nbk, 128)
                amax = blk.abs().amax(dim=(1, 3)).clamp_min(2.0 ** -126)
                sc = amax / 448.0
                q = torch.clamp(blk / sc[:, None, :, None], -448, 448).view(nbo * 128, nbk * 128)
                codes = q[:O_, :K_].to(torch.float8_e4m3fn)
            if keep is None or keep(name):
                out[name] = codes.view(torch.uint8).cpu().numpy()
                out[sname] = sc.float().cpu().numpy()
            i += 2
            continue
        if kind == "f32":
            if name.endswith("e_score_correction_bias"):
                v = torch.zeros(shape, device=dev)
            elif name.endswith("_scale"):
                v = 1.0 + 0.1 * torch.randn(shape, generator=g, device=dev)
            elif name.endswith("_base"):
                v = 0.25 * torch.randn(shape, generator=g, device=dev)
            else:                                   # A_log, dt_bias
                v = 0.5 * torch.randn(shape, generator=g, device=dev)
            out[name] = v.float().cpu().numpy()
        else:
            if len(shape) == 1 or name.endswith("compress_ape"):
                if name.endswith("bias") or name.endswith("compress_ape"):
                    v = 0.05 * torch.randn(shape, generator=g, device=dev)
                else:
                    v = 1.0 + 0.05 * torch.randn(shape, generator=g, device=dev)
            elif name in ("embed_tokens.weight", "lm_head.weight") or name.endswith("mlp.gate.weight"):
                v = 0.02 * torch.randn(shape, generator=g, device=dev)
            elif name.endswith("_conv1d.weight"):
                v = 0.25 * torch.randn(shape, generator=g, device=dev)
            else:
                v = torch.randn(shape, generator=g, device=dev) / math.sqrt(shape[-1])
            out[name] = bf16(v)
        i += 1
    if dev == "cuda":
        torch.cuda.empty_cache()
    return out
