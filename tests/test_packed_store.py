"""The packed-weight store: quantize once, save, reload and install without
the dense projection weights (structure and bytes on CPU; numerics on the GPU)."""
import pytest
import torch

from tests.conftest import load_kl
from tests.test_adapters import tiny_qwen

kl = load_kl()
transformers = pytest.importorskip("transformers")


def installed_tensors(model):
    out = {}
    for key, e in kl.export_packed(model)["entries"].items():
        for name in ("data", "scales", "zeros"):
            if e[name] is not None:
                out[f"{key}.{name}"] = e[name]
    return out


@pytest.mark.parametrize("fmt", ["w8_row", "w4_asym", "w4_sym"])
def test_round_trip_is_bit_exact(tmp_path, fmt):
    src = tiny_qwen(layers=3)
    kl.install_quantized_projections(src, fmt=fmt, layers=[0, 2], lm_head=fmt)
    path = tmp_path / "packed.pt"
    kl.save_packed(path, kl.export_packed(src))
    store = kl.load_packed(path)
    assert store["layers"] == {0: fmt, 2: fmt} and store["lm_head"] == fmt
    dst = tiny_qwen(layers=3, seed=1)                     # different dense weights: they must not be used
    info = kl.install_packed(dst, store)
    assert info["linear_modules"] == 15 and info["layers"] == {0: fmt, 2: fmt}
    a, b = installed_tensors(src), installed_tensors(dst)
    assert a.keys() == b.keys()
    for k in a:
        assert a[k].dtype == b[k].dtype and torch.equal(a[k], b[k]), k
    assert isinstance(dst.model.layers[1].self_attn.q_proj, torch.nn.Linear)      # layer 1 untouched


def test_install_on_meta_model_reads_no_dense_weight(tmp_path):
    src = tiny_qwen(layers=2)
    kl.install_quantized_projections(src, layers=[0, 1], lm_head="w8_row")
    path = tmp_path / "packed.pt"
    kl.save_packed(path, kl.export_packed(src))
    with torch.device("meta"):
        dst = transformers.Qwen3ForCausalLM(src.config)
    info = kl.install_packed(dst, kl.load_packed(path))
    assert info["dense_bytes_released"] == 0 and info["packed_bytes"] == src._kl_b200_info["packed_bytes"]
    assert dst.model.layers[1].self_attn.kl_qkv.weight_q.data.device.type == "cpu"
    # gate_proj / up_proj are row views of the packed gate_up matrix: no dense (meta) weight is left
    gp = dst.model.layers[0].mlp.gate_proj
    assert isinstance(gp, kl.adapters.RowSlice) and gp.weight.packed.data.device.type == "cpu"
    assert not any(p.device.type == "meta" for n, p in dst.named_parameters()
                   if ".layers." in n and ("_proj" in n))


def test_shape_and_plan_mismatches_raise(tmp_path):
    src = tiny_qwen(layers=2)
    kl.install_quantized_projections(src, layers=[0])
    store = kl.export_packed(src)
    wider = transformers.Qwen3Config(**{**src.config.to_dict(), "intermediate_size": 768})
    with pytest.raises(ValueError, match="gate_up"):
        kl.install_packed(transformers.Qwen3ForCausalLM(wider), store)
    with pytest.raises(ValueError, match="layer"):
        kl.install_packed(tiny_qwen(layers=2), dict(store, layers={5: "w8_row"}))
    missing = dict(store, entries={k: v for k, v in store["entries"].items() if not k.endswith(".down")})
    with pytest.raises(ValueError, match="no entry"):
        kl.install_packed(tiny_qwen(layers=2), missing)
    torch.save({"tag": "other"}, tmp_path / "x.pt")
    with pytest.raises(ValueError):
        kl.load_packed(tmp_path / "x.pt")


@pytest.mark.gpu
def test_loaded_model_matches_quantized_model(tmp_path):
    src = tiny_qwen(layers=2).cuda().to(torch.bfloat16)
    kl.install_quantized_projections(src, layers=[0, 1], lm_head="w8_row")
    path = tmp_path / "packed.pt"
    kl.save_packed(path, kl.export_packed(src))
    dst = tiny_qwen(layers=2).to(torch.bfloat16)              # same non-projection weights (same seed)
    kl.install_packed(dst, kl.load_packed(path, device="cuda"))
    dst = dst.cuda()
    ids = torch.randint(0, 1024, (1, 7), generator=torch.Generator().manual_seed(3)).cuda()
    with torch.no_grad():
        a = src(ids).logits
        b = dst(ids).logits
    torch.testing.assert_close(a, b, rtol=0, atol=0)
