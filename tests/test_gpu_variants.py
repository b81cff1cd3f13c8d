"""GPU tests of the variants kept beside the default lowerings.

The persistent attention schedule and the other attention variants kept for measurement, config 1's
one-division-per-row IR with the fast-math emitter options, and the unscheduled matmul nest lowered
to the tcgen05 GEMM.  Each is also checked on the CPU by the PTX / tensor-core emulators; here it is
compared with the oracle (or float64) on a B200.
"""
import pytest
import torch

from emmy_ptx_b200 import irgen, data
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph
from emmy_ptx_b200.runtime import Executable
from oracle.run import oracle_outputs
from tests.checks import compare, rtol_for
from tests.test_gpu_parity import _run_ours
from tests.test_gpu_parity import full_attention_check

pytestmark = pytest.mark.gpu


ATTN_VARIANTS = {
    "persistent-2ctas": {"attn_persistent": True, "sms": 2},
    "persistent-3ctas": {"attn_persistent": True, "sms": 3},
    "pack-in-turn": {"attn_pack_in_turn": True},
    "pack-after-turn": {"attn_pack_after_turn": True},
    "defer-sum": {"attn_pack_after_turn": True, "attn_defer_sum": True},
    "prefetch": {"attn_prefetch_next": 148},
    "poly8": {"attn_poly": 8},
    "f16-int4": {"attn_f16_int": 4},
    "no-turns": {"attn_pingpong": False},
    "bf16-pairs": {"attn_half": False},
    "pair-poly-2": {"attn_pair_poly": 2},
    "pair-poly-4": {"attn_pair_poly": 4},
    "kv128": {"attn_kv128": True},
    "kv128-ordered": {"attn_kv128": True, "attn_ordered": True},
    "kv128-bf16-pairs": {"attn_kv128": True, "attn_half": False},
    "kv128-pack-in-turn": {"attn_kv128": True, "attn_pack_in_turn": True},
}


_ORACLE_CACHE: dict = {}


def _small_with_oracle(key):
    """A small configuration's inputs and oracle outputs, computed once per key."""
    if key not in _ORACLE_CACHE:
        p = irgen.SMALL[key]()
        t = data.make_inputs(p)
        _ORACLE_CACHE[key] = (p, t, oracle_outputs(p, t))
    return _ORACLE_CACHE[key]


@pytest.mark.parametrize("key", ["c5tc", "c5tcnc"])
@pytest.mark.parametrize("variant", sorted(ATTN_VARIANTS))
def test_attention_variants_match_oracle(key, variant):
    """The opt-in attention variants (measured against the default for speed) give the default's
    results: each against the oracle on the small causal and non-causal configurations."""
    p, t, want = _small_with_oracle(key)
    got, ex = _run_ours(p, t, **ATTN_VARIANTS[variant])
    assert ex.records[-1]["kind"] == "tcgen05_attention"
    assert ex.error_code() == 0
    compare(got["O"], want["O"], "bf16", rtol_for(p), f"{key} {variant}", rms_floor=True)


def test_full_softmax_fast_math_options():
    """Config 1 in its measured variants: one division per row in the IR, and the opt-in approx_ftz
    and fast_div emitter options; all within the softmax tolerance at full size."""
    p = irgen.softmax_ir(4096, 1024, "warp", recip=True)
    t = data.make_inputs(p)
    want = torch.softmax(t["x"].cuda().double(), dim=-1).cpu()
    for opts in ({}, {"approx_ftz": True, "fast_div": True}):
        got, _ = _run_ours(p, t, **opts)
        compare(got["y"], want, "f32", 1e-5, f"c1 recip {opts}")


@pytest.mark.parametrize("opts", [{"attn_kv128": True}, {"attn_kv128": True, "attn_ordered": True}])
def test_full_attention_kv128_sampled(opts):
    """Config 5 at full size through the 128-row key/value block kernel; sampled heads against float64."""
    full_attention_check(opts)


def test_full_attention_persistent_sampled():
    """Config 5 at full size through the persistent schedule; sampled heads against float64."""
    full_attention_check({"attn_persistent": True})


def test_gemm_from_the_unscheduled_matmul():
    """The thread-per-element matmul nest, lowered to the tcgen05 GEMM, against the oracle."""
    p = irgen.bmm_naive_ir(2, 256, 512, 256)
    t = data.make_inputs(p)
    want = oracle_outputs(p, t)
    got, ex = _run_ours(p, t)
    assert ex.records[0]["kind"] == "tcgen05_gemm_pair" and ex.error_code() == 0
    compare(got["C"], want["C"], "f32", rtol_for(p), "bmm naive")
    got, ex = _run_ours(p, t, gemm_pair=False)
    assert ex.records[0]["kind"] == "tcgen05_gemm" and ex.error_code() == 0
    compare(got["C"], want["C"], "f32", rtol_for(p), "bmm naive, one CTA per tile")


@pytest.mark.parametrize("shape", [(2, 200, 264, 72), (1, 130, 8, 16), (3, 1000, 1000, 1000)])
def test_gemm_edge_tiles(shape):
    """The tcgen05 GEMM on shapes that are not tile multiples (edge tiles in M, N and K), against
    float64 with the matmul tolerance; the output is pre-filled with NaN so a row or column the
    kernel skips, or one it writes past, shows."""
    p = irgen.bmm_naive_ir(*shape)
    t = data.make_inputs(p)
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), {"gemm_pair": False})
    assert mod.kernels[0]["kind"] == "tcgen05_gemm"
    ex = Executable(mod)
    td = {k: v.cuda() for k, v in t.items()}
    b, m, n, _ = shape
    guard = torch.full((b * m * n + 4096,), float("nan"), dtype=torch.float32, device="cuda")
    td["C"] = guard[: b * m * n].view(b, m, n)
    ex(td)
    torch.cuda.synchronize()
    assert ex.error_code() == 0
    assert torch.isnan(guard[b * m * n:]).all(), "the kernel wrote past the output"
    want = t["A"].double() @ t["B"].double()
    compare(td["C"].cpu(), want, "f32", 1e-4, f"gemm edge {shape}")


@pytest.mark.parametrize("tma", [True, False])
def test_cuda_core_bmm_stripes(tma):
    """The CUDA-core batched matmul (tensor-core lowering off) with its operand stripes as TMA tile
    loads on mbarriers, and with the per-thread cp.async they replace, against float64."""
    p = irgen.bmm_ir(2, 512, 256, 384)
    t = data.make_inputs(p)
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), {"patterns": False, "tma_stripes": tma})
    assert ("cp.async.bulk.tensor" in mod.ptx) == tma
    ex = Executable(mod)
    td = {k: v.cuda() for k, v in t.items()}
    td["C"].fill_(float("nan"))
    ex(td)
    torch.cuda.synchronize()
    assert ex.error_code() == 0
    compare(td["C"].cpu(), t["A"].double() @ t["B"].double(), "f32", 1e-4, f"cuda-core bmm tma={tma}")


@pytest.mark.parametrize("causal", [True, False])
def test_attention_head_dim_64(causal):
    """Head dim 64 on the tensor cores: the small case against the oracle, and [2, 8, 2048, 64] against
    float64 on a few heads (first, middle and last)."""
    import math
    p = irgen.attention_ir(1, 2, 512, 64, causal)
    t = data.make_inputs(p)
    want = oracle_outputs(p, t)
    got, ex = _run_ours(p, t)
    assert ex.records[-1]["kind"] == "tcgen05_attention" and ex.error_code() == 0
    compare(got["O"], want["O"], "bf16", rtol_for(p), f"d64 causal={causal}", rms_floor=True)
    p = irgen.attention_ir(2, 8, 2048, 64, causal)
    t = data.make_inputs(p)
    got, ex = _run_ours(p, t)
    assert ex.error_code() == 0
    for b, h in ((0, 0), (1, 3), (1, 7)):
        q, k, v = (t[n][b, h].double() for n in ("Q", "K", "V"))
        s_ = (q @ k.T) / math.sqrt(64)
        if causal:
            s_ = s_.masked_fill(torch.ones_like(s_, dtype=torch.bool).triu(1), float("-inf"))
        compare(got["O"][b, h], torch.softmax(s_, -1) @ v, "bf16", 1e-4, f"d64 ({b},{h})", rms_floor=True)


@pytest.mark.parametrize("shape,causal", [((1, 2, 320, 128), True), ((1, 1, 200, 128), False),
                                          ((1, 4, 128, 64), False), ((2, 1, 300, 64), True)])
def test_attention_ragged_sequence(shape, causal):
    """S no multiple of 256 on the tensor cores: small cases against the oracle, and [1, 4, 1000, 128]
    (a partial last key block, rows past S that would land in the next head's rows if stored) against
    float64 on every head."""
    import math
    p = irgen.attention_ir(*shape, causal)
    t = data.make_inputs(p)
    want = oracle_outputs(p, t)
    got, ex = _run_ours(p, t)
    assert ex.records[-1]["kind"] == "tcgen05_attention" and ex.error_code() == 0
    compare(got["O"], want["O"], "bf16", rtol_for(p), f"ragged {shape} causal={causal}", rms_floor=True)
    p = irgen.attention_ir(1, 4, 1000, 128, causal)
    t = data.make_inputs(p)
    got, ex = _run_ours(p, t)
    assert ex.error_code() == 0
    for h in range(4):
        q, k, v = (t[n][0, h].double() for n in ("Q", "K", "V"))
        s_ = (q @ k.T) / math.sqrt(128)
        if causal:
            s_ = s_.masked_fill(torch.ones_like(s_, dtype=torch.bool).triu(1), float("-inf"))
        compare(got["O"][0, h], torch.softmax(s_, -1) @ v, "bf16", 1e-4, f"S=1000 head {h}", rms_floor=True)


@pytest.mark.parametrize("causal", [True, False])
def test_attention_explicit_mask(causal):
    """An explicit boolean mask on the tensor cores: the small case against the oracle (with rows whose
    first key blocks are all masked, and one row with every key masked: NaN, as in torch), and
    [1, 4, 1024, 128] with a random mask against float64 on every head."""
    import math
    p = irgen.attention_ir(1, 2, 256, 128, causal, mask=True)
    t = data.make_inputs(p)
    m = t["M"]
    m[7, :] = 0
    m[40:60, :128] = 0
    t["M"] = m
    want = oracle_outputs(p, t)
    got, ex = _run_ours(p, t)
    assert ex.records[-1]["kind"] == "tcgen05_attention" and ex.error_code() == 0
    compare(got["O"], want["O"], "bf16", rtol_for(p), f"mask causal={causal}", rms_floor=True)
    p = irgen.attention_ir(1, 4, 1024, 128, causal, mask=True)
    t = data.make_inputs(p)
    got, ex = _run_ours(p, t)
    assert ex.records[-1]["kind"] == "tcgen05_attention" and ex.error_code() == 0
    keep = t["M"].bool()
    for h in range(4):
        q, k, v = (t[n][0, h].double() for n in ("Q", "K", "V"))
        s_ = (q @ k.T) / math.sqrt(128)
        if causal:
            s_ = s_.masked_fill(torch.ones_like(s_, dtype=torch.bool).triu(1), float("-inf"))
        s_ = s_.masked_fill(~keep, float("-inf"))
        compare(got["O"][0, h], torch.softmax(s_, -1) @ v, "bf16", 1e-4, f"mask S=1024 head {h}", rms_floor=True)


def test_attention_explicit_mask_head_dim_64_ragged():
    """The mask with head dim 64 and S = 320 (a half-empty last query chunk) against the oracle."""
    p = irgen.attention_ir(1, 2, 320, 64, False, mask=True)
    t = data.make_inputs(p)
    want = oracle_outputs(p, t)
    got, ex = _run_ours(p, t)
    assert ex.records[-1]["kind"] == "tcgen05_attention" and ex.error_code() == 0
    compare(got["O"], want["O"], "bf16", rtol_for(p), "mask d64 S=320", rms_floor=True)


@pytest.mark.parametrize("shape,causal", [((1, 2, 64, 64), False), ((1, 2, 64, 64), True), ((1, 1, 48, 128), False),
                                          ((2, 3, 16, 64), True)])
def test_attention_shorter_than_one_tile(shape, causal):
    """S below one 128-row query tile on the tensor cores: the Q boxes and the last K/V box reach past the
    tensor and TMA reads zeros there; against the oracle."""
    p = irgen.attention_ir(*shape, causal)
    t = data.make_inputs(p)
    want = oracle_outputs(p, t)
    got, ex = _run_ours(p, t)
    assert ex.records[-1]["kind"] == "tcgen05_attention" and ex.error_code() == 0
    compare(got["O"], want["O"], "bf16", rtol_for(p), f"short {shape} causal={causal}", rms_floor=True)


@pytest.mark.parametrize("shape,causal", [((1, 2, 256, 32), True), ((1, 1, 320, 32), False), ((1, 4, 48, 32), False),
                                          ((2, 3, 16, 32), False)])
def test_attention_head_dim_32(shape, causal):
    """Head dim 32 on the tensor cores (64-byte rows, the 64-byte swizzle): small cases against the oracle,
    and [1, 4, 1024, 32] against float64 on every head."""
    import math
    p = irgen.attention_ir(*shape, causal)
    t = data.make_inputs(p)
    want = oracle_outputs(p, t)
    got, ex = _run_ours(p, t)
    assert ex.records[-1]["kind"] == "tcgen05_attention" and ex.error_code() == 0
    compare(got["O"], want["O"], "bf16", rtol_for(p), f"d32 {shape} causal={causal}", rms_floor=True)
    p = irgen.attention_ir(1, 4, 1024, 32, causal)
    t = data.make_inputs(p)
    got, ex = _run_ours(p, t)
    assert ex.error_code() == 0
    for h in range(4):
        q, k, v = (t[n][0, h].double() for n in ("Q", "K", "V"))
        s_ = (q @ k.T) / math.sqrt(32)
        if causal:
            s_ = s_.masked_fill(torch.ones_like(s_, dtype=torch.bool).triu(1), float("-inf"))
        compare(got["O"][0, h], torch.softmax(s_, -1) @ v, "bf16", 1e-4, f"d32 S=1024 head {h}", rms_floor=True)


@pytest.mark.parametrize("shape,causal", [((1, 2, 16, 32), False), ((1, 1, 80, 64), True), ((1, 1, 208, 128), False)])
def test_attention_mask_short_and_ragged(shape, causal):
    """The explicit mask with S a multiple of 16 but not of 64 (the reference's a_mask shape first), against
    the oracle: the last key block reads only the 16-byte mask pieces below S."""
    p = irgen.attention_ir(*shape, causal, mask=True)
    t = data.make_inputs(p)
    want = oracle_outputs(p, t)
    got, ex = _run_ours(p, t)
    assert ex.records[-1]["kind"] == "tcgen05_attention" and ex.error_code() == 0
    compare(got["O"], want["O"], "bf16", rtol_for(p), f"mask {shape}", rms_floor=True)


def test_attention_random_shapes_against_float64():
    """Twelve seeded random shapes (head dim 32, 64 or 128; S from 16 to 700; causal or not; a random
    mask where S allows it) on the tensor cores, each against float64 torch on every head."""
    import math
    import random
    rng = random.Random(20261202)
    for n in range(12):
        dim = rng.choice([32, 64, 128])
        seq = rng.choice([16, 48, 64, 96, 130, 200, 256, 320, 512, 700])
        causal = rng.random() < 0.5
        mask = seq % 16 == 0 and rng.random() < 0.4
        heads = rng.choice([1, 2, 3])
        p = irgen.attention_ir(1, heads, seq, dim, causal, mask=mask)
        t = data.make_inputs(p)
        got, ex = _run_ours(p, t)
        assert ex.records[-1]["kind"] == "tcgen05_attention" and ex.error_code() == 0, (dim, seq, causal, mask)
        for h in range(heads):
            q, k, v = (t[nm][0, h].double() for nm in ("Q", "K", "V"))
            s_ = (q @ k.T) / math.sqrt(dim)
            if causal:
                s_ = s_.masked_fill(torch.ones_like(s_, dtype=torch.bool).triu(1), float("-inf"))
            if mask:
                s_ = s_.masked_fill(~t["M"].bool(), float("-inf"))
            compare(got["O"][0, h], torch.softmax(s_, -1) @ v, "bf16", 1e-4,
                    f"random #{n} d{dim} S{seq} causal={causal} mask={mask} head {h}", rms_floor=True)
