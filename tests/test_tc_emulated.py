"""CPU parity of the tensor-core kernels: the emitted tcgen05 / TMA PTX run by the tensor-core emulator
(:mod:`tests.tcemu`) against the oracle, for the attention (default, variants, the value-range
fallback and the persistent schedule) and the batched matmul.

The GPU tests compare the same kernels on a B200; these also cover kernel forms that have not yet
run on a GPU, so their data path (descriptors, swizzled tiles, TMEM columns, row mapping) is checked
before any GPU time.
"""
import numpy as np
import pytest
import torch

from emmy_ptx_b200 import data, irgen
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph
from oracle.run import oracle_outputs
from tests.checks import compare, rms_floor_for, rtol_for
from tests.ptxemu import Memory
from tests.tcemu import TcEmulator
from tests.tcemu_pair import PairEmulator

_BYTES = {"f16": 2, "bf16": 2, "f32": 4, "i32": 4}


def _np(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()


def run_emulated(p, t, opts, defer=False, mod=None):
    """Compile ``p`` with ``opts`` (or take ``mod``) and run every entry through the emulator on
    tensors ``t``; returns the outputs and the error word."""
    mod = mod or compile_graph(Graph.from_dict(p.graph), p.meta(), opts)
    mem = Memory()
    addr = {name: mem.alloc(_np(ten).copy()) for name, ten in t.items()}
    for rec in mod.kernels:
        for spec in rec.get("scratch", []):
            if spec["name"] not in addr:
                addr[spec["name"]] = mem.alloc(np.zeros(int(np.prod(spec["shape"])) * _BYTES[spec["dtype"]], np.uint8))
    err = mem.alloc(np.zeros(16, np.uint8))
    for rec in mod.kernels:
        tm = {f"p_{spec['name']}": (addr[spec["tensor"]], spec) for spec in rec.get("tmaps", [])}
        cls = PairEmulator if list(rec.get("cluster", [1]))[0] == 2 else TcEmulator
        emu = cls(mod.ptx, rec["entry"], tm, defer=defer)
        plain = [q for q in emu.params if not q.startswith("p_tm") and q not in ("p_err", "p_trace")]
        args = dict(zip(plain, [addr[n] for n in rec["params"]]))
        args.update(emu.tmap_args())
        args["p_err"] = err
        emu.run(rec["grid"][0], rec["block"][0], args, mem, rec.get("dyn_smem", 0))
    out = {}
    for a in p.outputs:
        ten = t[a.name]
        arr = mem.array(addr[a.name], _np(ten).dtype, tuple(ten.shape)).copy()
        g = torch.from_numpy(arr)
        out[a.name] = g.view(torch.bfloat16) if ten.dtype == torch.bfloat16 else g
    return out, int(mem.array(err, np.int32, (4,))[0]), mod


def _check(p, t, opts, kind, defer=False, mod=None):
    got, code, mod = run_emulated(p, t, opts, defer, mod)
    assert mod.kernels[-1]["kind"] == kind
    assert code == 0
    want = oracle_outputs(p, t)
    for a in p.outputs:
        compare(got[a.name], want[a.name], a.dtype, rtol_for(p), f"tc-emu {opts}", rms_floor=rms_floor_for(p))


def _causal():
    # causal, one (batch, head), 512 rows: two work units (the longest first), so a persistent CTA
    # walks both, its warpgroups swapping the lower and upper rows between them
    return irgen.attention_ir(1, 1, 512, 128, True)


@pytest.mark.parametrize("key,opts", [
    ("c5tcnc", {}),
    ("c5tcnc", {"attn_half": False}),                  # P as two bf16 parts for every block
    ("c5tcnc", {"attn_pingpong": False}),
    ("causal", {}),
    ("causal", {"attn_persistent": True, "sms": 1}),
    ("c5tcnc", {"attn_persistent": True, "sms": 1}),
    ("c5tcnc", {"attn_prefetch_next": 1}),
    ("c5tcnc", {"attn_pack_in_turn": True}),
    ("c5tc", {"attn_persistent": True, "sms": 2}),        # 4 units over 2 CTAs: each walks a long and a short one
    ("c5tcnc", {"attn_pack_after_turn": True}),
    ("c5tcnc", {"attn_pack_after_turn": True, "attn_defer_sum": True}),
    ("c5tcnc", {"attn_poly": 8}),
    ("c5tcnc", {"attn_f16_int": 4}),
], ids=["nc", "nc-bf16", "nc-noturns", "causal", "causal-persistent", "nc-persistent", "nc-prefetch",
        "nc-pack-in-turn", "causal-persistent-2ctas", "nc-pack-after-turn", "nc-defer-sum", "nc-poly8",
        "nc-f16-int4"])
def test_attention_emulated_matches_oracle(key, opts):
    p = _causal() if key == "causal" else irgen.SMALL[key]()
    _check(p, data.make_inputs(p), opts, "tcgen05_attention")


@pytest.mark.parametrize("persistent", [False, True])
def test_attention_value_range_fallback_emulated(persistent):
    # one 64-row block of V scaled by 2^20 does not fit f16: that block takes the two-part bf16 path
    p = irgen.SMALL["c5tcnc"]()
    t = data.make_inputs(p)
    V = t["V"].float()
    V[:, :, 64:128] *= 2.0 ** 20
    t["V"] = V.to(torch.bfloat16)
    opts = {"attn_persistent": True, "sms": 1} if persistent else {}
    _check(p, t, opts, "tcgen05_attention")


@pytest.mark.parametrize("sms", [1, 2, 3])
def test_gemm_emulated_matches_oracle(sms):
    p = irgen.SMALL["c4tc"]()
    _check(p, data.make_inputs(p), {"sms": sms, "gemm_pair": False}, "tcgen05_gemm")


@pytest.mark.parametrize("key,opts", [
    ("nc512", {}),
    ("causal", {"attn_persistent": True, "sms": 1}),
    ("c5tcnc", {"attn_persistent": True, "sms": 1, "attn_half": False}),
], ids=["nc", "causal-persistent", "nc-persistent-bf16"])
def test_attention_with_late_completions(key, opts):
    # loads, MMAs and commits complete only when every thread waits, loads first, and the tensor core
    # advances only until a thread can run: a ring stage, Q tile, score buffer or O accumulator reused
    # before the hardware is done with it changes the result (8 kv blocks: every ring stage is reused)
    p = {"causal": _causal, "nc512": lambda: irgen.attention_ir(1, 1, 512, 128, False)}.get(
        key, lambda: irgen.SMALL[key]())()
    _check(p, data.make_inputs(p), opts, "tcgen05_attention", defer=True)


def test_gemm_with_late_completions():
    p = irgen.SMALL["c4tc"]()
    _check(p, data.make_inputs(p), {"sms": 2, "gemm_pair": False}, "tcgen05_gemm", defer=True)


def test_late_completions_expose_a_planted_early_release():
    # the ring's empty barriers wait for both issuers (count 2); with a count of 1 a stage is refilled
    # after the first issuer's MMAs, while the other tile's may still read it: with late completions
    # the run must fail (a wrong result, or the barrier accounting going wrong)
    import re
    from emmy_ptx_b200.compiler import CompiledModule
    from emmy_ptx_b200.kernels import tc_attention as ta
    p = irgen.attention_ir(1, 1, 512, 128, False)            # 8 kv blocks: every ring stage is reused
    t = data.make_inputs(p)
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), {})
    bad = mod.ptx
    for s_ in range(ta.STAGES):
        pat = r"(mbarrier\.init\.shared::cta\.b64 \[%r\d+\+" + str(ta.EMPTY + 8 * s_) + r"\]), 2;"
        bad, n = re.subn(pat, r"\1, 1;", bad)
        assert n == 1
    _check(p, t, {}, "tcgen05_attention", defer=True)            # the real kernel passes
    with pytest.raises((AssertionError, RuntimeError)):
        _check(p, t, {}, "tcgen05_attention", defer=True, mod=CompiledModule(bad, mod.kernels))


@pytest.mark.parametrize("causal,opts", [(True, {}), (False, {}), (True, {"attn_pingpong": False}),
                                         (True, {"attn_half": False})])
def test_attention_head_dim_64_emulated(causal, opts):
    """Head dim 64: a Q tile and a K/V block are one 64-column TMA box, PV has N=64 and O takes 64
    TMEM columns per tile."""
    p = irgen.attention_ir(1, 1, 512, 64, causal)
    _check(p, data.make_inputs(p), opts, "tcgen05_attention")


@pytest.mark.parametrize("shape", [(2, 32, 32, 64), (1, 200, 264, 72), (1, 130, 8, 16), (2, 128, 128, 96)])
def test_gemm_edge_tiles_emulated(shape):
    """Shapes that are not tile multiples: TMA zero-fills past M, N and K, the epilogue stores rows
    below M and 8-column groups below N (a store past the output would raise in the emulator)."""
    p = irgen.bmm_naive_ir(*shape)
    _check(p, data.make_inputs(p), {"gemm_pair": False}, "tcgen05_gemm")


def test_gemm_from_the_unscheduled_matmul_emulated():
    # the thread-per-element matmul nest lowered to the tcgen05 GEMM; the oracle interprets the nest
    p = irgen.bmm_naive_ir(1, 128, 256, 64)
    _check(p, data.make_inputs(p), {"sms": 1, "gemm_pair": False}, "tcgen05_gemm")


@pytest.mark.parametrize("shape,causal,opts", [
    ((1, 2, 320, 128), True, {}),                 # S % 64 == 0, not % 256: a half-empty last chunk
    ((1, 1, 200, 128), True, {}),                 # a partial last key block on the causal diagonal
    ((1, 1, 200, 128), False, {}),                # keys past S masked in the last block
    ((1, 2, 130, 64), False, {"attn_half": False}),
    ((1, 4, 128, 64), False, {}),                 # the reference's a_sdpa_big shape: tile 1 all past S
    ((2, 1, 300, 64), True, {"attn_pingpong": False}),
])
def test_attention_ragged_sequence_emulated(shape, causal, opts):
    """S no multiple of the 256-row query chunk: TMA zero-fills query and key rows past S, a full
    launch masks the keys past S, rows past S are not stored, and the value pre-pass neither reads
    nor writes past S (the emulator raises on an access outside an allocation)."""
    p = irgen.attention_ir(*shape, causal)
    _check(p, data.make_inputs(p), opts, "tcgen05_attention")


@pytest.mark.parametrize("shape,causal,opts", [
    ((1, 2, 256, 128), True, {}),
    ((1, 1, 256, 128), False, {"attn_half": False}),
    ((1, 1, 320, 64), False, {}),                 # the mask with a ragged sequence at head dim 64
])
def test_attention_explicit_mask_emulated(shape, causal, opts):
    """An explicit u8 mask [S, S] on the tensor cores: each softmax thread reads its row's 64 mask bytes
    per key block and masks the zero bytes (a random mask: half the keys of every row)."""
    p = irgen.attention_ir(*shape, causal, mask=True)
    _check(p, data.make_inputs(p), opts, "tcgen05_attention")


def test_attention_mask_with_fully_masked_blocks_and_rows():
    # rows whose first key blocks are all masked keep a running max of -inf and exponentiate against 0;
    # a row with every key masked is 0 / 0 = NaN, as in torch and in the IR's own semantics
    p = irgen.attention_ir(1, 1, 256, 128, False, mask=True)
    t = data.make_inputs(p)
    m = t["M"]
    m[5, :] = 0                                   # every key masked: NaN
    m[10:20, :128] = 0                            # the first two key blocks masked
    m[30, :] = 0
    m[30, 255] = 1                                # only the last key
    t["M"] = m
    _check(p, t, {}, "tcgen05_attention")


@pytest.mark.parametrize("shape,causal", [((1, 2, 64, 64), False), ((1, 2, 64, 64), True), ((1, 1, 48, 128), False),
                                          ((1, 1, 16, 64), True)])
def test_attention_shorter_than_one_tile_emulated(shape, causal):
    """S below one 128-row query tile (the reference's a_sdpa and a_sdpa_causal shapes): every Q box and
    the last K/V box reach past the tensor and read zeros there; the keys past S are masked."""
    p = irgen.attention_ir(*shape, causal)
    _check(p, data.make_inputs(p), {}, "tcgen05_attention")


@pytest.mark.parametrize("shape,causal,opts", [
    ((1, 2, 256, 32), True, {}),
    ((1, 1, 320, 32), False, {}),
    ((1, 1, 256, 32), True, {"attn_half": False}),
    ((1, 4, 48, 32), False, {}),                  # the reference's a_sdpa_scale shape (scale 1/sqrt(32) here)
    ((1, 2, 32, 32), False, {}),                  # a_sdpa_short
])
def test_attention_head_dim_32_emulated(shape, causal, opts):
    """Head dim 32: Q, K and V rows of 64 bytes, TMA boxes of 32 columns with the 64-byte swizzle, and
    SWIZZLE_64B shared-memory descriptors (K-major for Q and K, MN-major for V: one 32-column atom,
    16 rows of 64 bytes per MMA); PV has N=32 and O takes 32 TMEM columns per tile."""
    p = irgen.attention_ir(*shape, causal)
    _check(p, data.make_inputs(p), opts, "tcgen05_attention")


@pytest.mark.parametrize("shape,causal", [((1, 2, 16, 32), False), ((1, 1, 80, 64), True), ((1, 1, 208, 128), False)])
def test_attention_mask_short_and_ragged_emulated(shape, causal):
    """The explicit mask when S is a multiple of 16 but not of 64 (the reference's a_mask shape first):
    the last key block reads only its 16-byte mask pieces below S."""
    p = irgen.attention_ir(*shape, causal, mask=True)
    _check(p, data.make_inputs(p), {}, "tcgen05_attention")
