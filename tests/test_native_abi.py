"""CPU checks of the C ABI: the library loads, exports every symbol the header
declares, and the host-side launch planner partitions every BASELINE shape
correctly (no GPU needed)."""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

QWEN = [(4096, 1024), (1024, 2048), (6144, 1024), (1024, 3072), (151936, 1024)]
LLAMA = [(5120, 3072), (3072, 3072), (16384, 3072), (3072, 8192), (128256, 3072)]


def header_symbols():
    text = (ROOT / "include" / "kl_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(kl_\w+)\s*\(", text, re.M)))


def test_library_exports_every_header_symbol(kl):
    lib = kl._native.lib()
    declared = header_symbols()
    assert declared, "no declarations parsed from the header"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in kl_b200.h but not exported"
    assert set(declared) == set(kl._native.EXPORTED_SYMBOLS)
    assert lib.kl_version() >= 100


def test_status_strings(kl):
    lib = kl._native.lib()
    assert lib.kl_status_string(0) == b"ok"
    assert b"invalid" in lib.kl_status_string(1)
    assert b"workspace" in lib.kl_status_string(4)
    assert b"timed out" in lib.kl_status_string(5)


def test_validation_needs_no_gpu(kl):
    """Argument checks run before any CUDA call: bad shapes fail on a CPU box."""
    lib = kl._native.lib()
    N = kl._native
    # null pointers
    assert lib.kl_linear(None, 0, 1, 16, None, N.KL_W8_ROW, 16, 16, None, None, None, 0, None, None, 0, 0, None) == N.KL_ERR_INVALID
    assert b"non-null" in lib.kl_last_error()
    # reference op: warps must be 1/4/8, swiglu needs an even N
    fake = 256
    assert lib.kl_project(fake, 16, fake, 0, None, None, 8, 16, 2, 0, 0, fake, None, 0, None) == N.KL_ERR_INVALID
    assert b"warps" in lib.kl_last_error()
    assert lib.kl_project(fake, 16, fake, 0, None, None, 7, 16, 4, 0, 1, fake, None, 0, None) == N.KL_ERR_INVALID
    assert b"gate/up" in lib.kl_last_error()
    # int4 reference op: group and block_n domains
    assert lib.kl_int4_gemv(fake, 0, 128, fake, fake, 8, 48, 32, fake, None) == N.KL_ERR_INVALID
    assert lib.kl_int4_gemv(fake, 0, 128, fake, fake, 8, 128, 24, fake, None) == N.KL_ERR_INVALID


def prefill_tokens(m, n_tiles, sm=148):
    """Restatement of the pair kernel's token-tile choice: the tile count of
    each choice in waves over the CTA pairs, times max(tile tokens + 48, 192);
    the lowest cost wins, the larger tile on ties."""
    pairs = max(1, sm // 2)
    best, best_cost = 192, None
    for tok in (192, 128, 64):
        tiles = n_tiles * -(-m // tok)
        cost = -(-tiles // pairs) * max(tok + 48, 192)
        if best_cost is None or cost < best_cost:
            best, best_cost = tok, cost
    return best


def gemv_chain_plan(m, n, k, swiglu=False, sm=148, w4=False, group=128):
    """Restatement of the host planner of the CUDA-core chain GEMV (one or two
    tokens): about one CTA per SM with full rows, at most 64 output rows per
    CTA, shared memory padded to 80 KB so that at most two CTAs share an SM.
    4-bit rows take K/2 bytes plus an 8-byte (scale, zero) pair per group, and
    need a group that is a multiple of 16 dividing K, and K % 32 == 0."""
    if m > 2 or k % 16:
        return None
    if w4 and (group % 16 or k % group or k % 32):
        return None
    n_out = n // 2 if swiglu else n
    rows = -(-n_out // sm)
    mt = 1 if m <= 1 else 2
    # 4 rows per warp, or 8 above 32 rows per CTA (not for two-token SwiGLU)
    if rows > 64 or (rows > 32 and swiglu and mt == 2):
        return None
    h = 2 if swiglu else 1
    groups = h * rows * (k // group) * 8 if w4 else 0
    need = h * rows * (k // 2 if w4 else k) + ((groups + 15) // 16) * 16 + mt * k * 2 + 16
    if need > 227 * 1024:
        return None
    return {"rows": rows, "grid": -(-n_out // rows), "mt": mt, "smem": max(need, 80 * 1024),
            "rpw": 4 if rows <= 32 else 8}


def chain_plan(m, n, k, swiglu=False, sm=148):
    """Restatement of the host planner of the single-tile cluster kernel: the
    fewest 128-wide K blocks per CTA from 2 to 4 that keep the cluster portable
    (<= 8 CTAs) and the grid within one CTA per SM (two for 64-token tiles),
    else within two; None where it does not apply (M > 64, or a problem large
    enough for the persistent kernel)."""
    if m > 64:
        return None
    tiles = (n // 2 + 63) // 64 if swiglu else (n + 127) // 128
    kb = (k + 127) // 128
    caps = (2 * sm,) if m > 32 else (sm, 2 * sm)
    for cap in caps:
        for bpc in range(2, 5):
            csize = -(-kb // bpc)
            if csize <= 8 and tiles * csize <= cap:
                bpc = min(bpc, kb)
                return {"tiles": tiles, "bpc": bpc, "csize": -(-kb // bpc)}
    return None


@pytest.mark.parametrize("m", [1, 8, 16, 32, 64, 256, 512, 2048, 8192])
@pytest.mark.parametrize("n,k", QWEN + LLAMA)
def test_plan_partition_w8(kl, m, n, k):
    N = kl._native
    plan = N.describe_plan(m, n, k, N.KL_W8_ROW, sm_count=148)
    chain = chain_plan(m, n, k)
    gchain = gemv_chain_plan(m, n, k)
    # M >= 256 with K a multiple of 64 runs on the CTA-pair prefill kernel
    if m >= 256 and k % 64 == 0:
        assert plan["kernel"] == 3
        tok = prefill_tokens(m, (n + 255) // 256)
        assert plan["grid"] % 2 == 0 and plan["n_mma"] == tok and 1 <= plan["grid"] <= 148
        assert plan["tiles"] == ((n + 255) // 256) * ((m + tok - 1) // tok)
    elif gchain is not None:
        # one or two tokens: full rows per CTA on CUDA cores
        assert plan["kernel"] == 5
        assert (plan["grid"], plan["tiles"], plan["n_mma"], plan["smem"], plan["stages"]) == \
            (gchain["grid"], gchain["rows"], gchain["mt"], gchain["smem"], gchain["rpw"])
        assert plan["grid"] <= 148 and 80 * 1024 <= plan["smem"] <= 227 * 1024   # at most two CTAs per SM
        # the tcgen05 kernels stay available for the same problem (KL_FLAG_FORCE_TC)
        forced = N.describe_plan(m, n, k, N.KL_W8_ROW, flags=N.KL_FLAG_FORCE_TC, sm_count=148)
        assert forced["kernel"] == (4 if chain is not None else 2)
    elif chain is not None:
        # one decode linear small enough for the single-tile cluster kernel
        assert plan["kernel"] == 4
        assert plan["grid"] == chain["tiles"] * chain["csize"] <= 2 * 148 and chain["csize"] <= 8
        assert (plan["tiles"], plan["stages"], plan["units"]) == (chain["tiles"], chain["bpc"], chain["csize"])
        assert plan["n_mma"] == (16 if m <= 16 else 32 if m <= 32 else 64)
        # two CTAs per SM fit (shared memory) at two K blocks per CTA
        if plan["stages"] <= 2:
            assert 2 * plan["smem"] <= 228 * 1024
    else:
        assert plan["kernel"] == 2
    # the persistent stream-K kernel's plan, also taken with KL_FLAG_PERSISTENT
    if m <= 64:
        plan = N.describe_plan(m, n, k, N.KL_W8_ROW, flags=N.KL_FLAG_PERSISTENT, sm_count=148)
        assert plan["kernel"] == 2
        assert 1 <= plan["grid"] <= 148
        assert plan["smem"] <= 227 * 1024
        assert plan["n_mma"] in (16, 32, 64)
        assert plan["stages"] >= 3          # weight ring of >= 3 stages (16-32 KB each) per SM


def test_chain_plan_config1_shapes(kl):
    """Clusters of the Qwen3-0.6B decode linears: QKV splits K four ways (2
    blocks per CTA), o eight ways (2 blocks), down eight ways (3 blocks);
    gate_up three ways (3 blocks, 144 CTAs) up to 32 tokens and four ways (2
    blocks, 192 CTAs) for 64-token tiles; the lm_head is too large and streams
    through the persistent kernel."""
    N = kl._native
    expect = {(4096, 1024, False): (32, 4, 4), (1024, 2048, False): (8, 8, 8), (6144, 1024, True): (48, 3, 4),
              (1024, 3072, False): (8, 8, 8)}
    for (n, k, sw), (tiles, csize, csize64) in expect.items():
        for m in (1, 8, 32, 64):
            plan = N.describe_plan(m, n, k, N.KL_W8_ROW, swiglu=sw, flags=N.KL_FLAG_FORCE_TC, sm_count=148)
            want = csize64 if m > 32 else csize
            assert plan["kernel"] == 4 and (plan["tiles"], plan["units"]) == (tiles, want), (n, k, m, plan)
    assert N.describe_plan(1, 151936, 1024, N.KL_W8_ROW, sm_count=148)["kernel"] == 2


@pytest.mark.parametrize("m", [1, 16, 64, 512, 8192])
@pytest.mark.parametrize("n,k", [(6144, 1024), (12288, 1024), (16384, 3072)])
def test_plan_partition_swiglu(kl, m, n, k):
    plan = kl._native.describe_plan(m, n, k, kl._native.KL_W8_ROW, swiglu=True, sm_count=148)
    if m >= 256:
        tok = prefill_tokens(m, (n // 2 + 127) // 128)
        assert plan["kernel"] == 3 and plan["n_mma"] == tok
        assert plan["tiles"] == ((n // 2 + 127) // 128) * ((m + tok - 1) // tok)
    elif gemv_chain_plan(m, n, k, swiglu=True) is not None:
        assert plan["kernel"] == 5 and plan["tiles"] == gemv_chain_plan(m, n, k, swiglu=True)["rows"]
    elif chain_plan(m, n, k, swiglu=True) is not None:
        assert plan["kernel"] == 4 and plan["tiles"] == (n // 2 + 63) // 64
    else:
        assert plan["kernel"] == 2 and plan["tiles"] == ((n // 2 + 63) // 64) * ((m + plan["n_mma"] - 1) // plan["n_mma"])


@pytest.mark.parametrize("m", [1, 2, 16, 200])
@pytest.mark.parametrize("n,k", QWEN)
def test_plan_partition_w4(kl, m, n, k):
    N = kl._native
    for fmt in (N.KL_W4_ASYM, N.KL_W4_SYM):
        plan = N.describe_plan(m, n, k, fmt, sm_count=148)
        g = gemv_chain_plan(m, n, k, w4=True)
        if g is not None:
            # one or two tokens: the CUDA-core chain GEMV with full 4-bit rows
            assert plan["kernel"] == 5
            assert (plan["grid"], plan["tiles"], plan["n_mma"], plan["smem"]) == (g["grid"], g["rows"], g["mt"], g["smem"])
            assert N.describe_plan(m, n, k, fmt, flags=N.KL_FLAG_PERSISTENT, sm_count=148)["kernel"] == 2
        else:
            assert plan["kernel"] == 2 and plan["n_mma"] <= 64


def test_plan_w4_two_group_stages(kl):
    """Two 128-groups per stage (256-wide K blocks) only where the stage can
    carry its zero points: asymmetric 4-bit needs K % 1024 == 0 (16-byte rows
    of bf16 zeros for the TMA box); symmetric 4-bit has no zeros and needs
    K % 256 == 0."""
    N = kl._native
    tiles = (151936 + 127) // 128
    assert N.describe_plan(1, 151936, 2048, N.KL_W4_ASYM)["units"] == tiles * 2048 // 256
    assert N.describe_plan(1, 151936, 1280, N.KL_W4_ASYM)["units"] == tiles * 1280 // 128
    assert N.describe_plan(1, 151936, 1280, N.KL_W4_SYM)["units"] == tiles * 1280 // 256
    # ~128 KB of weights in flight per SM: a zero-carrying stage is 16 KB of
    # nibbles + 2 KB of zeros, so the ring holds one stage fewer
    asym = N.describe_plan(1, 151936, 2048, N.KL_W4_ASYM)
    sym = N.describe_plan(1, 151936, 2048, N.KL_W4_SYM)
    assert asym["threads"] == sym["threads"] == 512
    assert sym["stages"] == 128 * 1024 // 16384 and asym["stages"] == 128 * 1024 // (16384 + 2048)
    assert asym["smem"] <= 227 * 1024 and sym["smem"] <= 227 * 1024


@pytest.mark.parametrize("sm", [1, 7, 132, 148, 296])
def test_plan_partition_odd_grids(kl, sm):
    for n, k in [(17, 128), (1024, 1024), (151936, 1024)]:
        kl._native.describe_plan(3, n, k, kl._native.KL_W8_ROW, sm_count=sm)


def test_simt_plan_for_reference_formats(kl):
    N = kl._native
    assert N.describe_plan(1, 34, 256, N.KL_W8_GROUP)["kernel"] == 1
    assert N.describe_plan(1, 33, 7, N.KL_BF16_DENSE)["kernel"] == 1
    assert N.describe_plan(1, 17, 128, N.KL_W4_SYM, flags=N.KL_FLAG_FORCE_SIMT)["kernel"] == 1


def test_prefill_token_tiles_fill_the_pairs():
    """The N = 1024 GEMMs of a 2048-token prefill take 128-token tiles (64 tiles
    for 74 pairs instead of 44 at 192); the wide ones keep 192."""
    N_ = None
    from tests.conftest import load_kl
    N_ = load_kl()._native
    assert N_.describe_plan(2048, 1024, 2048, N_.KL_W8_ROW, sm_count=148)["n_mma"] == 128
    assert N_.describe_plan(2048, 1024, 3072, N_.KL_W8_ROW, sm_count=148)["n_mma"] == 128
    assert N_.describe_plan(8192, 4096, 1024, N_.KL_W8_ROW, sm_count=148)["n_mma"] == 192
    assert N_.describe_plan(8192, 1024, 2048, N_.KL_W8_ROW, sm_count=148)["n_mma"] == 192
    assert N_.describe_plan(2048, 4096, 1024, N_.KL_W8_ROW, sm_count=148)["n_mma"] == 192
    assert N_.describe_plan(512, 1024, 2048, N_.KL_W8_ROW, sm_count=148)["n_mma"] == 128
