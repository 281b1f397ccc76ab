"""The weight-container reader (include/apus_gmtp_gcuda.h: config_load,
container_check, container_read) on the host, no GPU: both config layouts
the reference's loader accepts (c/gmodel.h:373-480), a container written in
the reference's layout, error reports for a missing or mistyped tensor, and,
when the reference tree is present in this container, the reference's own
real config.json and a container made by the reference's converter from its
own synthetic checkpoint (tests/m1/fixtures.py + tools/convert.py)."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from container import write_container
from modelgen import gen_weights, tiny_config

REF = "/root/reference"


@pytest.fixture(scope="module")
def G():
    import apus_gcuda
    return apus_gcuda


def _kw_fields(G, kw):
    return {k: kw[k] for k, _ in G._CFG_FIELDS if k not in ("layer_is_dsa", "mlp_is_sparse")}


def test_flat_config_round_trip(G, tmp_path):
    kw = tiny_config()
    W = gen_weights(kw, seed=5)
    cfgp = write_container(str(tmp_path), kw, W, G.tensor_specs(kw))
    got = G.config_dict(G.config_load(cfgp))
    for k, v in _kw_fields(G, kw).items():
        assert got[k] == pytest.approx(v), k
    assert got["layer_is_dsa"] == list(kw["layer_is_dsa"])
    assert got["mlp_is_sparse"] == list(kw["mlp_is_sparse"])


def test_nested_config_layout(G, tmp_path):
    """The real checkpoint's layout: text_config, KDA keys inside
    linear_attn_config, booleans, explicit layer lists overriding the rule."""
    kw = tiny_config(num_hidden_layers=6, first_k_dense_replace=2)
    tc = _kw_fields(G, kw)
    for k in ("linear_num_heads", "linear_head_dim", "linear_conv_kernel_dim", "linear_lower_bound"):
        tc.pop(k)
    tc["linear_attn_config"] = {"num_heads": 2, "head_dim": 128, "short_conv_kernel_size": 4,
                                "gate_lower_bound": -5.0}
    tc["norm_topk_prob"] = True
    tc["index_kpool_always_select_tail"] = False
    tc["layer_types"] = ["linear_attention", "deepseek_sparse_attention"] * 3
    (tmp_path / "config.json").write_text(json.dumps({"model_type": "glm5_next", "text_config": tc}))
    got = G.config_dict(G.config_load(str(tmp_path / "config.json")))
    assert got["linear_num_heads"] == 2 and got["linear_head_dim"] == 128
    assert got["linear_conv_kernel_dim"] == 4 and got["linear_lower_bound"] == -5.0
    assert got["norm_topk_prob"] == 1 and got["index_kpool_always_select_tail"] == 0
    assert got["layer_is_dsa"] == [0, 1, 0, 1, 0, 1]              # the explicit list
    assert got["mlp_is_sparse"] == [0, 0, 1, 1, 1, 1]             # the rule (no list given)


def test_config_errors(G, tmp_path):
    (tmp_path / "bad.json").write_text('{"hidden_size": 4096')
    with pytest.raises(G.GcudaError):
        G.config_load(str(tmp_path / "bad.json"))
    (tmp_path / "short.json").write_text('{"hidden_size": 4096}')
    with pytest.raises(G.GcudaError, match="missing"):
        G.config_load(str(tmp_path / "short.json"))


@pytest.mark.skipif(not os.path.exists(os.path.join(REF, "reference", "config.json")),
                    reason="the reference tree is not present")
def test_reference_real_config(G):
    c = G.config_dict(G.config_load(os.path.join(REF, "reference", "config.json")))
    assert (c["hidden_size"], c["num_hidden_layers"], c["vocab_size"]) == (4096, 45, 154880)
    assert (c["linear_num_heads"], c["linear_head_dim"], c["linear_conv_kernel_dim"]) == (64, 128, 4)
    assert c["num_nextn_predict_layers"] == 1 and c["n_routed_experts"] == 288
    assert c["layer_is_dsa"] == [int(i % 4 == 3) for i in range(45)]
    assert c["mlp_is_sparse"] == [int(i >= 3) for i in range(45)]


def test_container_check_and_read(G, tmp_path):
    kw = tiny_config()
    W = gen_weights(kw, seed=6)
    specs = G.tensor_specs(kw)
    write_container(str(tmp_path), kw, W, specs, n_shards=3)
    cfg = G.make_config(**kw)
    assert G.container_check(str(tmp_path), cfg, True) == len(specs)
    for name, _, _, _ in specs:
        assert G.container_read(str(tmp_path), name) == np.ascontiguousarray(W[name]).tobytes(), name


def test_container_errors(G, tmp_path):
    kw = tiny_config()
    W = gen_weights(kw, seed=7)
    specs = G.tensor_specs(kw)
    cfg = G.make_config(**kw)
    # a missing tensor
    missing = specs[5][0]
    write_container(str(tmp_path / "a"), kw, W, [s for s in specs if s[0] != missing])
    with pytest.raises(G.GcudaError, match="no tensor " + missing.replace(".", r"\.")):
        G.container_check(str(tmp_path / "a"), cfg, True)
    # a tensor stored with the wrong dtype
    bad = [(n, sh, dt, "f32" if n == "norm.weight" else k) for n, sh, dt, k in specs]
    W2 = dict(W)
    W2["norm.weight"] = np.zeros(kw["hidden_size"], np.float32)
    write_container(str(tmp_path / "b"), kw, W2, bad)
    with pytest.raises(G.GcudaError, match="norm.weight is F32"):
        G.container_check(str(tmp_path / "b"), cfg, True)
    with pytest.raises(G.GcudaError):
        G.container_check(str(tmp_path / "nowhere"), cfg, True)


def _fixture_kw():
    """The model config of the reference's M1 fixture checkpoint."""
    m1 = os.path.join(REF, "tests", "m1")
    sys.path.insert(0, m1)
    try:
        import fixtures as F
    finally:
        sys.path.remove(m1)
    return dict(hidden_size=F.H, vocab_size=F.VOCAB, num_hidden_layers=F.N_LAYERS_MAIN, rms_norm_eps=1e-5,
                hc_mult=F.HC, hc_sinkhorn_iters=20, hc_eps=1e-6, first_k_dense_replace=3,
                intermediate_size=F.DENSE_INTER, moe_intermediate_size=F.MOE_INTER, n_routed_experts=F.N_EXPERTS,
                n_shared_experts=1, num_experts_per_tok=2, routed_scaling_factor=2.5, norm_topk_prob=1,
                swiglu_limit=10.0, num_attention_heads=F.N_HEADS, q_lora_rank=F.Q_LORA, kv_lora_rank=F.KV_LORA,
                qk_nope_head_dim=F.QD, v_head_dim=F.VD, index_n_heads=F.I_HEADS, index_head_dim=F.I_DIM,
                index_topk=8, index_kpool=F.KPOOL, index_kpool_always_select_tail=1,
                linear_num_heads=F.LIN_HEADS, linear_head_dim=F.LIN_DIM, linear_conv_kernel_dim=F.CONV_K,
                linear_lower_bound=-5.0, num_nextn_predict_layers=1,
                layer_is_dsa=[int(i in F.DSA_LAYERS) for i in range(F.N_LAYERS_MAIN)],
                mlp_is_sparse=[int(i in F.MOE_LAYERS) for i in range(F.N_LAYERS_MAIN)])


def _converted(tmp_path):
    """A container made by the reference converter from its own synthetic
    checkpoint (tests/m1/fixtures.py + tools/convert.py), and the config."""
    m1 = os.path.join(REF, "tests", "m1")
    src, dst = tmp_path / "src", tmp_path / "dst"
    src.mkdir()
    code = ("import sys; sys.path.insert(0, %r); import fixtures; fixtures.make_fixture_tree(%r)" % (m1, str(src)))
    subprocess.check_call([sys.executable, "-c", code])
    subprocess.check_call([sys.executable, os.path.join(REF, "tools", "convert.py"), "convert", str(src), str(dst)],
                          stdout=subprocess.DEVNULL)
    return src, dst


@pytest.mark.skipif(not os.path.exists(os.path.join(REF, "tools", "convert.py")),
                    reason="the reference tree is not present")
def test_manifest_checks(G, tmp_path):
    """The v2 manifest apus.index.json (c/gmodel.h:647-660, c/gcache.h:865-930)
    is checked against the shards: a tampered version, tensor offset, slab
    size or slab member order is refused with the reason."""
    import shutil
    _, dst = _converted(tmp_path)
    cfg = G.make_config(**_fixture_kw())
    assert G.container_check(str(dst), cfg, True) > 0
    man = json.load(open(dst / "apus.index.json"))
    name = next(iter(man["tensor_map"]))

    def tampered(tag, edit):
        d = tmp_path / tag
        shutil.copytree(dst, d)
        m = json.loads(json.dumps(man))
        edit(m)
        (d / "apus.index.json").write_text(json.dumps(m))
        return str(d)

    cases = [
        ("v1", lambda m: m.update(format_version=1), "not a glm5_next v2 container"),
        ("off", lambda m: m["tensor_map"][name].update(offset=m["tensor_map"][name]["offset"] + 8),
         "disagrees with the shards for " + name.replace(".", r"\.")),
        ("slab", lambda m: m["expert_slabs"][0].update(nbytes=m["expert_slabs"][0]["nbytes"] + 4), "size"),
        ("order", lambda m: m.update(expert_slab_members=list(reversed(m["expert_slab_members"]))),
         "laid end to end"),
    ]
    for tag, edit, msg in cases:
        with pytest.raises(G.GcudaError, match=msg):
            G.container_check(tampered(tag, edit), cfg, True)


@pytest.mark.skipif(not os.path.exists(os.path.join(REF, "tools", "convert.py")),
                    reason="the reference tree is not present")
def test_reference_converter_container(G, tmp_path):
    """The reference converter's own output (byte-identical repack, expert
    slabs, split experts reassembled, vision stripped, MTP shard group) reads
    back through this reader with every tensor the model needs and the same
    bytes as the reference's source checkpoint."""
    m1 = os.path.join(REF, "tests", "m1")
    src, dst = _converted(tmp_path)
    sys.path.insert(0, m1)
    try:
        import fixtures as F
        import stutil
    finally:
        sys.path.remove(m1)
    kw = _fixture_kw()
    cfg = G.make_config(**kw)
    n = G.container_check(str(dst), cfg, True)
    # every source tensor of the language model, by its container name
    src_map = json.load(open(src / "model.safetensors.index.json"))["weight_map"]
    lang = {k: v for k, v in src_map.items() if not k.startswith(F.VIS)}
    assert n == len(lang)
    src_bytes = {}
    for shard in sorted(set(lang.values())):
        src_bytes.update(stutil.read_tensor_bytes(os.path.join(src, shard)))
    for name in lang:
        cname = name[len(F.LANG):] if name.startswith(F.LANG) else name
        assert G.container_read(str(dst), cname) == src_bytes[name], cname
