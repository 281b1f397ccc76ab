"""A model loaded from a weight container in the reference's layout
(apus_gcuda_config_load + apus_gcuda_model_load_container) is bitwise the
model loaded tensor by tensor with apus_gcuda_model_set: same decode logits,
same speculative stream, same committed state."""
import numpy as np
import pytest

from container import write_container
from modelgen import gen_weights, tiny_config

pytestmark = pytest.mark.gpu

PROMPT = [5, 17, 300, 2, 99, 42, 7, 381, 0, 11, 13]


def test_container_model_equals_set_model(gcuda, tmp_path):
    kw = tiny_config()
    W = gen_weights(kw, seed=20261202)
    cfg_path = write_container(str(tmp_path), kw, W, gcuda.tensor_specs(kw), n_shards=3)
    cfg = gcuda.config_load(cfg_path)
    a = gcuda.GModel(cfg, has_mtp=True, kv_cap=256, depth=4)
    a.load_container(str(tmp_path))
    b = gcuda.GModel(gcuda.make_config(**kw), has_mtp=True, kv_cap=256, depth=4)
    b.load(W)
    ids = np.array(PROMPT[:6], np.int32)
    assert np.array_equal(a.decode_batch(ids), b.decode_batch(ids))
    for m in (a, b):
        m.reset()
        m.spec_prefill(PROMPT)
    sa, sb = [], []
    for _ in range(6):
        sa += a.spec_step()
        sb += b.spec_step()
    assert sa == sb and a.digest() == b.digest()
    # a tensor read back from the device equals the container's bytes
    got = a.get("layers.3.mlp.experts.3.down_proj.weight", W["layers.3.mlp.experts.3.down_proj.weight"].shape,
                np.uint8)
    assert np.array_equal(got, W["layers.3.mlp.experts.3.down_proj.weight"])
    a.close()
    b.close()


def test_container_load_errors(gcuda, tmp_path):
    kw = tiny_config()
    W = gen_weights(kw, seed=3)
    specs = gcuda.tensor_specs(kw)
    write_container(str(tmp_path), kw, W, [s for s in specs if not s[0].startswith("layers.2.mlp.gate_proj")])
    m = gcuda.GModel(gcuda.make_config(**kw), has_mtp=True, kv_cap=64, depth=2)
    with pytest.raises(gcuda.GcudaError, match="layers.2.mlp.gate_proj"):
        m.load_container(str(tmp_path))
    m.close()
