"""The dense-contraction matcher: what it accepts and what it must refuse (CPU only)."""
import copy
import json

from emmy_ptx_b200 import irgen
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph
from emmy_ptx_b200.patterns import match_bmm, match_attention


def _kernel(p):
    g = Graph.from_dict(p.graph)
    return g, g.kernels()[0]


def test_bmm_ir_is_recognised_as_a_contraction():
    for p in (irgen.FULL["c4"](), irgen.SMALL["c4tc"](), irgen.SMALL["c4"]()):
        g, k = _kernel(p)
        hit = match_bmm(g, k)
        assert hit is not None
        X, Y, C, bt, m, n, kk = hit
        assert (X.name, Y.name, C.name) == ("A", "B", "C")
        assert (bt, m, n, kk) == (p.params["batch"], p.params["m"], p.params["n"], p.params["k"])


def test_tile_multiples_select_the_tensor_core_kernel():
    p = irgen.FULL["c4"]()
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), {"gemm_pair": False})
    rec = mod.kernels[0]
    assert rec["kind"] == "tcgen05_gemm" and rec["entry"] == "bmm_bf16"
    assert rec["params"] == ["A", "B", "C"] and rec["block"] == [192, 1, 1]
    pair = compile_graph(Graph.from_dict(p.graph), p.meta()).kernels[0]
    assert pair["kind"] == "tcgen05_gemm_pair" and pair["cluster"] == [2, 1, 1] and pair["grid"] == [148, 1, 1]
    for ins in ("tcgen05.mma.cta_group::1.kind::f16", "tcgen05.alloc", "tcgen05.dealloc",
                "cp.async.bulk.tensor.3d", "tcgen05.ld.sync.aligned.32x32b.x32", "mbarrier.try_wait.parity"):
        assert ins in mod.ptx
    assert "multicast" not in mod.ptx
    small = irgen.SMALL["c4"]()          # N = 128, half of the 256-wide tile: one edge tile in N
    assert compile_graph(Graph.from_dict(small.graph), small.meta()).kernels[0]["kind"] == "tcgen05_gemm_pair"
    odd_k = irgen.bmm_naive_ir(1, 64, 64, 36)     # K % 8 != 0: A's rows are no whole 16-byte TMA units
    assert compile_graph(Graph.from_dict(odd_k.graph), odd_k.meta()).kernels[0]["kind"] == "generic"
    odd_n = irgen.bmm_naive_ir(1, 64, 20, 64)     # N % 8 != 0: B's rows likewise
    assert compile_graph(Graph.from_dict(odd_n.graph), odd_n.meta()).kernels[0]["kind"] == "generic"


def test_swapped_contraction_axis_is_refused():
    p = irgen.SMALL["c4tc"]()
    d = copy.deepcopy(p.graph)
    body = d["nodes"]["bmm_bf16"]["op_fields"]["body"][2]["body"]
    kloop = next(st for st in body if st["kind"] == "StridedLoop")
    cond = next(st for st in kloop["body"] if st["kind"] == "Cond")
    copy_a = next(st for st in cond["body"] if st["src"] == "A")
    copy_a["src_index"][1], copy_a["src_index"][2] = copy_a["src_index"][2], copy_a["src_index"][1]
    g = Graph.from_dict(d)
    assert match_bmm(g, g.kernels()[0]) is None


def test_non_product_accumulation_is_refused():
    p = irgen.SMALL["c4tc"]()
    d = copy.deepcopy(p.graph)

    def edit(stmts):
        for st in stmts:
            if st.get("kind") == "Assign" and st.get("name") == "p00":
                st["op"]["name"] = "add"
            for key in ("body", "else_body"):
                if isinstance(st.get(key), list):
                    edit(st[key])
    edit(d["nodes"]["bmm_bf16"]["op_fields"]["body"])
    g = Graph.from_dict(d)
    assert match_bmm(g, g.kernels()[0]) is None


def test_patterns_can_be_disabled():
    p = irgen.FULL["c4"]()
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), {"patterns": False})
    assert mod.kernels[0]["kind"] == "generic"


def test_attention_ir_is_recognised():
    for key, tab, causal in (("c5", irgen.FULL, True), ("c5tc", irgen.SMALL, True), ("c5tcnc", irgen.SMALL, False)):
        p = tab[key]()
        g, k = _kernel(p)
        hit = match_attention(g, k)
        assert hit is not None, key
        Q, K, V, O, bt, hd, seq, dim, c, scale, M = hit
        assert M is None
        assert (Q.name, K.name, V.name, O.name) == ("Q", "K", "V", "O")
        assert (bt, hd, seq, dim, c) == (p.params["batch"], p.params["heads"], p.params["seq"], p.params["dim"], causal)
        assert abs(scale - p.params["scale"]) < 1e-7
    full = irgen.FULL["c5"]()
    one = compile_graph(Graph.from_dict(full.graph), full.meta()).kernels
    assert [r["kind"] for r in one] == ["value_prepass", "tcgen05_attention"] and one[1]["grid"] == [4096, 1, 1]
    assert one[1]["block"] == [384, 1, 1]
    recs = compile_graph(Graph.from_dict(full.graph), full.meta(), {"attn_overlap": True}).kernels
    # opt-in: the pre-pass of 7/8 of the (batch, head) pairs runs on the side stream beside the
    # attention of the first 1/8; the grids add up to the whole problem
    assert [r["kind"] for r in recs] == ["value_prepass", "tcgen05_attention"] * 2
    assert [r.get("stream", 0) for r in recs] == [0, 0, 1, 0]
    assert recs[2]["after"] == [recs[0]["entry"]] and recs[3]["after"] == [recs[2]["entry"]]
    assert recs[3]["entry"] == "attention_causal"
    for rec in recs[1::2]:
        assert rec["block"] == [384, 1, 1]
    assert recs[1]["grid"][0] + recs[3]["grid"][0] == 4096 and recs[1]["grid"][0] == 512
    assert recs[0]["grid"][0] == 32 * 64 and recs[2]["grid"][0] == 148      # the side pre-pass strides


def test_attention_with_a_different_mask_is_refused():
    p = irgen.SMALL["c5tc"]()
    d = copy.deepcopy(p.graph)

    def edit(stmts):
        for st in stmts:
            if st.get("kind") == "Select":
                st["branches"][0]["select"]["op"] = ">="          # excludes the diagonal: not causal
            for key in ("body", "else_body"):
                if isinstance(st.get(key), list):
                    edit(st[key])
    edit(d["nodes"]["attention_causal"]["op_fields"]["body"])
    g = Graph.from_dict(d)
    assert match_attention(g, g.kernels()[0]) is None


def test_small_head_dim_stays_on_cuda_cores():
    # head dim 256 has no tensor-core form; 32, 64 and 128 do, at any S
    p = irgen.attention_ir(1, 1, 16, 256, False)
    assert compile_graph(Graph.from_dict(p.graph), p.meta()).kernels[0]["kind"] == "generic"
    d32 = irgen.attention_ir(1, 2, 64, 32, False)
    assert compile_graph(Graph.from_dict(d32.graph), d32.meta()).kernels[-1]["kind"] == "tcgen05_attention"
    short = irgen.SMALL["c5nc"]()             # D = 64, S = 32: below one query tile, on the tensor cores
    assert compile_graph(Graph.from_dict(short.graph), short.meta()).kernels[-1]["kind"] == "tcgen05_attention"


def _mutated(p, entry, edit):
    d = copy.deepcopy(p.graph)

    def visit(stmts):
        for st in stmts:
            edit(st)
            for key in ("body", "else_body"):
                if isinstance(st.get(key), list):
                    visit(st[key])
    visit(d["nodes"][entry]["op_fields"]["body"])
    g = Graph.from_dict(d)
    return g, g.kernels()[0]


def _swap_first_write_values():
    done = []

    def edit(st):
        if st.get("kind") == "Write" and not done:
            st["values"][0], st["values"][1] = st["values"][1], st["values"][0]
            done.append(st)
    return edit


def test_bmm_near_misses_are_refused():
    # each of these passed the structural checks alone: a store to C[b, j, i] and two accumulators
    # written to each other's places would have produced a wrong C from the tensor-core kernel
    p = irgen.SMALL["c4tc"]()

    def transpose_store(st):
        if st.get("kind") == "Write":
            st["index"][1], st["index"][2] = st["index"][2], st["index"][1]
    for edit in (transpose_store, _swap_first_write_values()):
        g, k = _mutated(p, "bmm_bf16", edit)
        assert match_bmm(g, k) is None, edit.__name__
        assert compile_graph(g, p.meta()).kernels[0]["kind"] == "generic"


def test_attention_near_misses_are_refused():
    p = irgen.SMALL["c5tc"]()

    def shared_kv_head(st):                       # K[b, 0, kv, d]: every head reads head 0's keys
        if st.get("kind") == "Load" and st.get("input") == "K":
            st["index"][1] = {"kind": "Literal", "value": 0, "dtype": "i32"}

    def v_transposed(st):                         # V[b, h, d, kv]
        if st.get("kind") == "Load" and st.get("input") == "V":
            st["index"][2], st["index"][3] = st["index"][3], st["index"][2]
    for edit in (shared_kv_head, v_transposed, _swap_first_write_values()):
        g, k = _mutated(p, "attention_causal", edit)
        assert match_attention(g, k) is None, edit.__name__
        assert [r["kind"] for r in compile_graph(g, p.meta()).kernels] == ["generic"], edit.__name__


def test_attention_with_another_scale_is_lowered_with_it():
    # the softmax scale is a kernel parameter: a nest with another scale literal is still the
    # canonical nest for that scale
    p = irgen.SMALL["c5tc"]()

    def other_scale(st):
        if st.get("kind") == "Assign" and st.get("name") == "sc":
            st["args"][1]["value"] = 0.1
    g, k = _mutated(p, "attention_causal", other_scale)
    hit = match_attention(g, k)
    assert hit is not None and abs(hit[9] - 0.1) < 1e-9


def test_renamed_buffers_still_match():
    # the equality gate compares bodies up to the buffer names
    p = irgen.SMALL["c4tc"]()
    d = copy.deepcopy(p.graph)
    blob = json.dumps(d).replace('"A"', '"lhs"').replace('"B"', '"rhs"').replace('"C"', '"out"')
    g = Graph.from_dict(json.loads(blob))
    hit = match_bmm(g, g.kernels()[0])
    assert hit is not None and (hit[0].name, hit[1].name, hit[2].name) == ("lhs", "rhs", "out")


def test_unscheduled_matmul_reaches_the_tensor_cores():
    # a thread per output element with a rolled k loop is the same contraction: it takes the tcgen05
    # GEMM (edge tiles where M or N is not a tile multiple); with K % 8 != 0, or a transposed store,
    # it stays on the CUDA cores
    p = irgen.bmm_naive_ir(1, 128, 256, 64)
    g, k = _kernel(p)
    assert match_bmm(g, k) is not None
    assert compile_graph(g, p.meta()).kernels[0]["kind"] == "tcgen05_gemm_pair"
    edge = irgen.bmm_naive_ir(1, 100, 256, 64)
    g1, _ = _kernel(edge)
    assert compile_graph(g1, edge.meta()).kernels[0]["kind"] == "tcgen05_gemm_pair"
    odd = irgen.bmm_naive_ir(1, 100, 256, 60)
    g2, k2 = _kernel(odd)
    assert compile_graph(g2, odd.meta()).kernels[0]["kind"] == "generic"

    def transpose_store(st):
        if st.get("kind") == "Write":
            st["index"][1], st["index"][2] = st["index"][2], st["index"][1]
    g3, k3 = _mutated(p, "bmm_naive", transpose_store)
    assert match_bmm(g3, k3) is None


def _rename_locals(p, entry, keep):
    """Every SSA name of the kernel (not the buffers in ``keep``, not an operator or type) prefixed
    with ``t_``: the same program under other local names."""
    d = copy.deepcopy(p.graph)
    semantic = {"kind", "dtype", "value_dtype", "swizzle", "op"}

    def go(v, key=None, kind=None):
        if isinstance(v, str):
            if key in semantic or (key == "name" and kind in ("ElementwiseImpl", "ReduceOp", "Builtin")) or v in keep:
                return v
            return "t_" + v
        if isinstance(v, list):
            return [go(x, key, kind) for x in v]
        if isinstance(v, dict):
            return {k: go(x, k, v.get("kind")) for k, x in v.items()}
        return v
    body = d["nodes"][entry]["op_fields"]["body"]
    d["nodes"][entry]["op_fields"]["body"] = go(body)
    g = Graph.from_dict(d)
    return g, g.kernels()[0]


def test_renamed_locals_and_commuted_products_still_match():
    # the gate compares bodies up to local value names and the operand order of commutative f32
    # operations: an Emmy lowering that names its values differently still reaches the tensor cores
    p = irgen.SMALL["c4tc"]()
    g, k = _rename_locals(p, "bmm_bf16", {"A", "B", "C"})
    assert match_bmm(g, k) is not None
    assert compile_graph(g, p.meta()).kernels[0]["kind"] == "tcgen05_gemm_pair"

    def commute(st):
        if st.get("kind") == "Assign" and st["op"]["name"] == "multiply":
            st["args"].reverse()
    g, k = _mutated(p, "bmm_bf16", commute)
    assert match_bmm(g, k) is not None
    q = irgen.SMALL["c5tc"]()
    g, k = _rename_locals(q, "attention_causal", {"Q", "K", "V", "O"})
    assert match_attention(g, k) is not None
    assert compile_graph(g, q.meta()).kernels[-1]["kind"] == "tcgen05_attention"


def test_commuting_a_subtraction_is_refused():
    # operand order matters for subtract: exp(m - s) is not exp(s - m)
    p = irgen.SMALL["c5tc"]()

    def flip(st):
        if st.get("kind") == "Assign" and st["op"]["name"] == "subtract":
            st["args"].reverse()
    g, k = _mutated(p, "attention_causal", flip)
    assert match_attention(g, k) is None
    assert [r["kind"] for r in compile_graph(g, p.meta()).kernels] == ["generic"]
