"""Mirror of the reference's learning/09_int4/test_int4.py against the B200 ops."""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as O
from tests.conftest import load_kl

kl = load_kl()


@pytest.mark.parametrize('group', [32, 64, 128])
def test_pack_roundtrip_cpu(group):
    w = torch.arange(-7, 8, dtype=torch.float32).repeat(group)[:group].repeat(3, 1)
    packed = kl.quantize_int4(w, group_size=group, chunk_rows=2)
    torch.testing.assert_close(kl.dequantize_int4(packed), w, rtol=0, atol=0)
    assert packed.storage_bytes == w.numel() // 2 + 3 * 4


def test_zero_groups_and_invalid_input():
    p = kl.quantize_int4(torch.zeros(2, 128))
    assert torch.equal(kl.dequantize_int4(p), torch.zeros(2, 128))
    assert torch.isfinite(p.scales).all()
    with pytest.raises(ValueError):
        kl.quantize_int4(torch.ones(2, 127))
    with pytest.raises(ValueError):
        kl.quantize_int4(torch.full((2, 128), float('nan')))


@pytest.mark.parametrize('group', [32, 64, 128])
def test_quantization_error_bound(group):
    torch.manual_seed(5)
    w = torch.randn(7, 256)
    packed = kl.quantize_int4(w, group)
    bound = packed.scales.repeat_interleave(group, -1) / 2 + 1e-6
    assert ((w - kl.dequantize_int4(packed)).abs() <= bound).all()


@pytest.mark.parametrize('group', [32, 64, 128])
def test_cpu_packer_matches_reference_bits(golden, group):
    p = kl.quantize_int4(torch.from_numpy(golden[f"i4_err{group}_w"]), group)
    np.testing.assert_array_equal(p.data.numpy(), golden[f"i4_err{group}_data"])
    np.testing.assert_array_equal(p.scales.numpy(), golden[f"i4_err{group}_scales"])


@pytest.mark.gpu
@pytest.mark.parametrize('group', [32, 64, 128])
def test_gpu_packer_matches_reference_bits(golden, group):
    p = kl.quantize_int4(torch.from_numpy(golden[f"i4_err{group}_w"]).cuda(), group)
    np.testing.assert_array_equal(p.data.cpu().numpy(), golden[f"i4_err{group}_data"])
    np.testing.assert_array_equal(p.scales.cpu().numpy(), golden[f"i4_err{group}_scales"])
    torch.testing.assert_close(kl.dequantize_native(p).cpu(), torch.from_numpy(golden[f"i4_err{group}_deq"]),
                               rtol=0, atol=0)


@pytest.mark.gpu
@pytest.mark.parametrize('dtype', [torch.float16, torch.bfloat16])
@pytest.mark.parametrize('n,k', [(17, 128), (1024, 1024), (2048, 1024), (3072, 1024), (1024, 3072)])
def test_gemv_against_dequantized_oracle(dtype, n, k):
    torch.manual_seed(42)
    w = torch.randn(n, k, device='cuda', dtype=dtype) / k ** .5
    x = torch.randn(k, device='cuda', dtype=dtype)
    packed = kl.quantize_int4(w)
    expected = (kl.dequantize_int4(packed) @ x.float()).to(dtype)
    actual = kl.int4_gemv(x, packed)
    torch.testing.assert_close(actual, expected, rtol=.02, atol=.002)


@pytest.mark.gpu
@pytest.mark.parametrize('n', [17, 65, 151936])
@pytest.mark.parametrize('top', [1, 4, 8])
def test_fused_head_selection(n, top):
    torch.manual_seed(13)
    w = torch.randn(n, 128, device='cuda', dtype=torch.bfloat16) / 128 ** .5
    x = torch.randn(128, device='cuda', dtype=w.dtype)
    packed = kl.quantize_int4(w)
    logits = kl.int4_gemv(x, packed).float()
    scores, ids = kl.int4_lm_head_topk(x, packed, top_k=top)
    torch.testing.assert_close(scores, logits.topk(top).values, rtol=0, atol=0)
    torch.testing.assert_close(scores, logits[ids], rtol=0, atol=0)
    assert ids.unique().numel() == top
    if top == 1:
        assert ids.item() == logits.argmax().item()


@pytest.mark.gpu
def test_argmax_tie():
    p = kl.quantize_int4(torch.zeros(65, 128, device='cuda', dtype=torch.bfloat16))
    _, ids = kl.int4_lm_head_topk(torch.ones(128, device='cuda', dtype=torch.bfloat16), p)
    assert ids.item() == 0


@pytest.mark.gpu
def test_head_golden(golden):
    g = golden
    packed = kl.PackedInt4(torch.from_numpy(g["i4_head_data"]).cuda(), torch.from_numpy(g["i4_head_scales"]).cuda(), 128)
    x = torch.from_numpy(g["i4_head_x"]).bfloat16().cuda()
    logits = kl.int4_gemv(x, packed).float().cpu().numpy()
    assert (np.abs(logits - g["i4_head_logits"]) <= np.maximum(2 ** -8, np.abs(g["i4_head_logits"]) * 2 ** -7)).all()
    for top in (1, 4, 8):
        v, i = kl.int4_lm_head_topk(x, packed, top_k=top)
        ov, oi = O.topk_lowest_index(logits, top)
        np.testing.assert_array_equal(v.cpu().numpy(), ov)
        np.testing.assert_array_equal(i.cpu().numpy(), oi)
