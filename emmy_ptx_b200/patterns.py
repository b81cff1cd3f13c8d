"""Tensor-core lowering of dense-contraction Accum loop nests.

The IR schedules a batched matmul for CUDA cores (cp.async stripes into shared memory, a
register micro-tile of ``Accum(add, multiply(a, b))``).  When a kernel provably computes

    C[b, i, j] = sum_k X[b, i, k] * Y[b, k, j]      (X, Y bf16, C f32)

it is emitted as the tcgen05/TMA kernel of :mod:`.kernels.tc_gemm` instead.  The match is
structural and fails closed — anything not recognised exactly is left to the CUDA-core path:

* exactly two inputs and one output; shapes [B,M,K] x [B,K,N] -> [B,M,N]; dtypes bf16/bf16/f32;
* every shared buffer is filled by CpAsyncCopy from exactly one input, one buffer per input;
* inside the K loop, the copy from X indexes X's last axis with the loop counter and Y's middle
  axis with it (and the other axes without it) — the contraction axis is K on both sides;
* every Accum is ``add`` of a product of one value loaded from X's buffer and one from Y's,
  seeded with 0; every Write goes to the output and writes only accumulators; nothing else is
  written to global memory;
* the GEMM's N and K are multiples of 8 (16-byte TMA rows; partial 128 x 256 edge tiles are
  zero-filled on load and clipped on store); attention has head dim 32, 64 or 128 and any S (rows
  and keys past S in the last 256-row query chunk are zero-filled, masked and not stored; that holds for
  S below one tile too).

Those checks find the operands, shapes and (for attention) the mask and scale.  The final gate is
stricter: the kernel body must equal the canonical CUDA-core nest for those parameters
(:func:`.irgen.bmm_ir`, :func:`.irgen.bmm_naive_ir`, :func:`.irgen.attention_ir`), up to the buffer
names, the names of local values and the operand order of commutative f32 operations.  A structural check alone let a
store to C[b, j, i] or two swapped accumulators through; with the equality gate no variation of the
nest can reach a tensor-core kernel that computes something else, and every other form runs, correctly,
on the CUDA cores.
"""
from __future__ import annotations

import json
import os

from .ir import Graph, dt_name, walk


def _body_data(node, rename=None) -> list:
    """The kernel body as plain data, with every string equal to a key of ``rename`` mapped."""
    def ren(v):
        if isinstance(v, str):
            return rename.get(v, v)
        if isinstance(v, list):
            return [ren(x) for x in v]
        if isinstance(v, dict):
            return {k: ren(x) for k, x in v.items()}
        return v
    data = [st.to_dict() for st in node.op.body]
    return ren(data) if rename else data


# Strings the IR gives meaning to (everything else a bare string holds is an SSA or buffer name):
# class names, types, operator spellings, and the names of elementwise / reduction / builtin /
# called functions.
_SEMANTIC_KEYS = frozenset({"kind", "dtype", "value_dtype", "swizzle", "op"})
_SEMANTIC_NAME = frozenset({"ElementwiseImpl", "ReduceOp", "Builtin", "FuncCallExpr"})
_COMMUTATIVE = frozenset({"add", "multiply", "maximum", "minimum"})


def _alpha(data, fixed: frozenset):
    """``data`` with every SSA name replaced by its rank of first appearance, buffer names in
    ``fixed`` kept, and the two arguments of a commutative Assign in a canonical order.  Two bodies
    equal after this differ only in what they call their local values (and the operand order of
    f32 add / multiply / max / min, which IEEE arithmetic does not depend on), so they compute the
    same thing."""
    names: dict[str, str] = {}

    def canon(v: str) -> str:
        if v in fixed:
            return v
        if v not in names:
            names[v] = f"%{len(names)}"
        return names[v]

    def go(v, key=None, kind=None):
        if isinstance(v, str):
            if key in _SEMANTIC_KEYS or (key == "name" and kind in _SEMANTIC_NAME) or (
                    key == "value" and kind in ("Literal", "Dim")):
                return v
            return canon(v)
        if isinstance(v, list):
            return [go(x, key, kind) for x in v]
        if isinstance(v, dict):
            k2 = v.get("kind")
            out = {k: go(x, k, k2) for k, x in v.items()}
            if (k2 == "Assign" and isinstance(v.get("op"), dict) and v["op"].get("name") in _COMMUTATIVE
                    and len(out.get("args") or []) == 2):
                out["args"] = sorted(out["args"], key=lambda a: json.dumps(a, sort_keys=True))
            return out
        return v
    return go(data)


def is_canonical(node, template, rename: dict) -> bool:
    """True when ``node``'s body, its buffers renamed by ``rename``, equals the body of the single
    kernel of ``template`` (a problem from :mod:`.irgen`, or a callable making one: a generator that
    has no form for these parameters raises ValueError, and then nothing matches), up to the names
    of local values and the operand order of commutative f32 operations."""
    if callable(template):
        try:
            template = template()
        except ValueError:
            return False
    tnode = Graph.from_dict(template.graph).kernels()[0]
    fixed = frozenset(rename.values()) | frozenset(tnode.inputs) | frozenset(v.name for v in tnode.outputs)
    return _alpha(_body_data(node, rename), fixed) == _alpha(_body_data(tnode), fixed)


def _names_in(e, out: set) -> set:
    """Every variable name an index expression mentions."""
    if e is None:
        return out
    if isinstance(e, str):
        out.add(e)
        return out
    if isinstance(e, (list, tuple)):
        for x in e:
            _names_in(x, out)
        return out
    cls = type(e).__name__
    if cls == "Var":
        out.add(e.name)
    for attr in ("left", "right", "cond", "if_true", "if_false", "expr"):
        v = getattr(e, attr, None)
        if v is not None and not isinstance(v, (int, float)):
            _names_in(v, out)
    for attr in ("args", "index"):
        for v in getattr(e, attr, None) or ():
            _names_in(v, out)
    return out


def _closure(names: set, deps: dict) -> set:
    out = set()
    stack = list(names)
    while stack:
        n = stack.pop()
        if n in out:
            continue
        out.add(n)
        stack.extend(deps.get(n, ()))
    return out


def match_bmm(graph, node):
    """(X, Y, C, batch, M, N, K) when the kernel is a batched bf16 matmul, else None."""
    op = node.op
    vals = graph.values()
    if len(node.outputs) != 1 or len(node.inputs) != 2:
        return None
    C = node.outputs[0]
    ins = [vals.get(n) for n in node.inputs]
    if any(v is None for v in ins):
        return None
    if dt_name(C.dtype) != "f32" or len(C.shape) != 3:
        return None
    if any(dt_name(v.dtype) != "bf16" or len(v.shape) != 3 for v in ins):
        return None
    bt, m, n = C.shape
    X = next((v for v in ins if v.shape[0] == bt and v.shape[1] == m), None)
    Y = next((v for v in ins if v is not X and v.shape[0] == bt and v.shape[2] == n), None)
    if X is None or Y is None or X.shape[2] != Y.shape[1]:
        return None
    k = X.shape[2]
    rename = {X.name: "A", Y.name: "B", C.name: "C"}
    from .irgen import bmm_ir, bmm_naive_ir
    if is_canonical(node, lambda: bmm_naive_ir(bt, m, n, k), rename):
        return X, Y, C, bt, m, n, k              # the unscheduled nest: one thread per element

    stmts = []
    walk(op.body, stmts.append)
    deps: dict[str, set] = {}
    for st in stmts:
        cls = type(st).__name__
        if cls == "Let":
            deps[st.name] = _names_in(st.value, set())
        elif cls == "Assign":
            deps[st.name] = _names_in(list(st.args), set())
    # shared buffers and their single global source
    src_of: dict[str, set] = {}
    for st in stmts:
        if type(st).__name__ == "CpAsyncCopy":
            src_of.setdefault(st.smem, set()).add(st.src)
    if any(len(v) != 1 for v in src_of.values()):
        return None
    feeds = {next(iter(v)): s for s, v in src_of.items()}
    if set(feeds) != {X.name, Y.name} or len(src_of) != 2:
        return None
    sX, sY = feeds[X.name], feeds[Y.name]
    # the K loop: the loop whose body copies stripes; its counter must index the contraction axis
    kloops = []
    walk(op.body, lambda st: kloops.append(st) if type(st).__name__ in ("StridedLoop", "Loop") and any(
        type(s).__name__ == "CpAsyncCopy" for s in _flat(st.body)) else None)
    if len(kloops) != 1:
        return None
    kname = kloops[0].axis.name
    for st in _flat(kloops[0].body):
        if type(st).__name__ != "CpAsyncCopy":
            continue
        idx = list(st.src_index)
        if len(idx) != 3:
            return None
        dep = [kname in _closure(_names_in(x, set()), deps) for x in idx]
        if st.src == X.name and dep != [False, False, True]:
            return None
        if st.src == Y.name and dep != [False, True, False]:
            return None
    # loads from the shared buffers, products, accumulators
    loaded = {}
    for st in stmts:
        if type(st).__name__ == "Load" and st.input in (sX, sY):
            for nm in st.names:
                loaded[nm] = st.input
    products = {}
    for st in stmts:
        if type(st).__name__ == "Assign" and (getattr(st.op, "name", None) or str(st.op)) == "multiply":
            args = list(st.args)
            if len(args) == 2 and all(isinstance(x, str) for x in args):
                srcs = {loaded.get(args[0]), loaded.get(args[1])}
                if srcs == {sX, sY}:
                    products[st.name] = True
    accs = set()
    for st in stmts:
        cls = type(st).__name__
        if cls == "Accum":
            if (getattr(st.op, "name", None) or str(st.op)) != "add" or getattr(st, "base", None) not in (None, st.name):
                return None
            if not isinstance(st.value, str) or st.value not in products:
                return None
            accs.add(st.name)
    if not accs:
        return None
    for st in stmts:
        cls = type(st).__name__
        if cls == "Init" and st.name in accs and float(st.identity) != 0.0:
            return None
        if cls == "Write":
            if st.output in src_of:
                continue
            if st.output != C.name or getattr(st, "atomic", False):
                return None
            if not all(v in accs for v in st.values):
                return None
        if cls == "ZeroPrologue":
            return None
    if not is_canonical(node, lambda: bmm_ir(bt, m, n, k), rename):
        return None
    return X, Y, C, bt, m, n, k


def _is_var(e, name=None) -> bool:
    return type(e).__name__ == "Var" and (name is None or e.name == name)


def _index_vars(index) -> list:
    """Variable names per coordinate of an index list (None where a coordinate is not a lone Var)."""
    out = []
    for e in index:
        if isinstance(e, str):
            out.append(e)
        elif _is_var(e):
            out.append(e.name)
        else:
            out.append(None)
    return out


def match_attention(graph, node):
    """(Q, K, V, O, batch, heads, seq, dim, causal, scale, M) when the kernel is the online-softmax
    attention nest, else None; M is the explicit u8 mask [S, S] or None.

    Recognised form (the attention IR): a Tile over (b, h, q, lane); Q loaded at [b, h, q, d0]; one
    kv loop from 0 to S with step 1 whose body loads K and V at [b, h, kv, d0], reduces the lane
    products of Q and K with an ``add`` WarpShuffle, multiplies by a float literal (the scale), masks
    with a Select whose first branch is ``kv > q -> -inf`` (causal) or has no mask, keeps the running
    max as ``Accum(maximum)`` and the row sum / output as ``Accum(add, base=...)``; after the loop
    every written value is ``divide(o, l)`` to O at [b, h, q, d0].  With an explicit mask the kv
    loop also loads M at [q, kv] and masks a zero byte to -inf."""
    op = node.op
    vals = graph.values()
    if len(node.outputs) != 1 or len(node.inputs) not in (3, 4):
        return None
    O = node.outputs[0]
    if dt_name(O.dtype) != "bf16" or len(O.shape) != 4:
        return None
    bt, hd, seq, dim = O.shape
    ins = [vals.get(n) for n in node.inputs]
    if any(v is None for v in ins):
        return None
    M = None
    if len(ins) == 4:
        masks = [v for v in ins if dt_name(v.dtype) == "u8" and tuple(v.shape) == (seq, seq)]
        if len(masks) != 1:
            return None
        M = masks[0]
        ins = [v for v in ins if v is not M]
    if any(dt_name(v.dtype) != "bf16" or tuple(v.shape) != tuple(O.shape) for v in ins):
        return None
    tiles = [st for st in op.body if type(st).__name__ == "Tile"]
    if len(tiles) != 1 or len(tiles[0].axes) != 4:
        return None
    tile = tiles[0]
    ax = [a.name for a in tile.axes]
    from .ir import dim_int
    if [dim_int(a.extent) for a in tile.axes] != [bt, hd, seq, 32] or dim % 32:
        return None
    stmts = []
    walk(op.body, stmts.append)
    loops = [st for st in stmts if type(st).__name__ in ("StridedLoop", "Loop")]
    if len(loops) != 1 or type(loops[0]).__name__ != "StridedLoop":
        return None
    lp = loops[0]
    kv = lp.axis.name
    if lp.start != 0 or lp.step != 1 or (lp.end if lp.end is not None else dim_int(lp.axis.extent)) != seq:
        return None
    inner = []
    walk(lp.body, inner.append)
    loads_in = {st.input: st for st in inner if type(st).__name__ == "Load"}
    if M is not None:
        if M.name not in loads_in:
            return None
        loads_in.pop(M.name)             # its form ([q, kv], a zero byte -> -inf) is the canonical check's
    loads_out = [st for st in stmts if type(st).__name__ == "Load" and st not in inner]
    if len(loads_in) != 2 or len(loads_out) != 1:
        return None
    qload = loads_out[0]
    Q = vals.get(qload.input)
    kv_inputs = [n for n in loads_in if n != qload.input]
    if Q is None or len(kv_inputs) != 2:
        return None
    d0 = _index_vars(qload.index)[3]
    if _index_vars(qload.index)[:3] != ax[:3] or d0 is None:
        return None
    for ld in loads_in.values():
        if _index_vars(ld.index) != [ax[0], ax[1], kv, d0]:
            return None
    shuffles = [st for st in inner if type(st).__name__ == "WarpShuffle"]
    if len(shuffles) != 1 or shuffles[0].length != 32:
        return None
    comb = list(shuffles[0].combine_states or ())
    if len(comb) != 1 or (getattr(comb[0].op, "name", None) or str(comb[0].op)) != "add":
        return None
    dot = shuffles[0].state[0]
    # which loaded input meets Q in the dot product: K; the other one feeds the output Accums: V
    assign = {st.name: st for st in stmts if type(st).__name__ == "Assign"}
    qnames = set(qload.names)

    def sources(name, seen=None):
        seen = set() if seen is None else seen
        if name in seen:
            return set()
        seen.add(name)
        out = set()
        for ld in list(loads_in.values()) + [qload]:
            if name in ld.names:
                out.add(ld.input)
        a = assign.get(name)
        if a is not None:
            for x in a.args:
                if isinstance(x, str):
                    out |= sources(x, seen)
        return out

    dsrc = sources(dot)
    if Q.name not in dsrc:
        return None
    kname = next((n for n in kv_inputs if n in dsrc), None)
    vname = next((n for n in kv_inputs if n != kname), None)
    if kname is None or vname is None or vname in dsrc:
        return None
    scale = None
    for st in inner:
        if type(st).__name__ == "Assign" and (getattr(st.op, "name", None) or str(st.op)) == "multiply":
            args = list(st.args)
            if len(args) == 2 and args[0] == dot and type(args[1]).__name__ == "Literal":
                scale = float(args[1].value)
    if scale is None:
        return None
    sels = [st for st in inner if type(st).__name__ == "Select"]
    causal = False
    if len(sels) > (2 if M is not None else 1):
        return None
    for sel in sels:
        br = sel.branches[0]
        c = br.select
        v = br.value
        if (type(c).__name__ == "BinaryExpr" and c.op == ">" and _is_var(c.left, kv) and _is_var(c.right, ax[2])
                and type(v).__name__ == "Literal" and float(v.value) == float("-inf")):
            causal = True                # the first branch masks kv > q: causal (the canonical check
            #                              below confirms every branch)
    accs = [st for st in inner if type(st).__name__ == "Accum"]
    ops = sorted((getattr(a.op, "name", None) or str(a.op)) for a in accs)
    if ops.count("maximum") != 1 or ops.count("add") != 1 + dim // 32:
        return None
    writes = [st for st in stmts if type(st).__name__ == "Write"]
    if len(writes) != 1 or writes[0].output != O.name or _index_vars(writes[0].index) != [ax[0], ax[1], ax[2], d0]:
        return None
    for v in writes[0].values:
        a = assign.get(v)
        if a is None or (getattr(a.op, "name", None) or str(a.op)) != "divide":
            return None
    K = vals[kname]
    V = vals[vname]
    from .irgen import attention_ir
    rename = {Q.name: "Q", K.name: "K", V.name: "V", O.name: "O", **({M.name: "M"} if M is not None else {})}
    if not is_canonical(node, lambda: attention_ir(bt, hd, seq, dim, causal, scale=scale, mask=M is not None),
                        rename):
        return None
    return Q, K, V, O, bt, hd, seq, dim, causal, scale, M


def _flat(body):
    out = []
    walk(body, out.append)
    return out


def try_lower(graph, node, kmeta, prefix, options):
    """A tensor-core build record for this kernel, or None to keep the CUDA-core lowering."""
    if options.get("patterns") is False or os.environ.get("EMMY_B200_PATTERNS", "1") == "0":
        return None
    hit = match_bmm(graph, node)
    if hit is not None:
        X, Y, C, bt, m, n, k = hit
        from .kernels import tc_gemm
        if not tc_gemm.supported(m, n, k):
            return None
        if options.get("gemm_pair", True):
            # CTA pairs (the default; 16 % faster on config 4): 256 x 256 tiles from
            # tcgen05.mma.cta_group::2 (kernels/tc_gemm_pair.py); gemm_pair=False keeps one CTA per tile
            from .kernels import tc_gemm_pair
            return tc_gemm_pair.gemm_pair_entry(node.op.name, bt, m, n, k, pairs=int(options.get("sms", 148)) // 2,
                                                names=(X.name, Y.name, C.name), prefix=prefix,
                                                stages=int(options.get("gemm_stages", tc_gemm_pair.STAGES)))
        b = tc_gemm.gemm_entry(node.op.name, bt, m, n, k, sms=int(options.get("sms", 148)),
                               names=(X.name, Y.name, C.name), prefix=prefix)
        return b
    hit = match_attention(graph, node)
    if hit is not None:
        Q, K, V, O, bt, hd, seq, dim, causal, scale, M = hit
        from .kernels import tc_attention
        if dim not in (32, 64, 128):
            return None
        if M is not None and seq % 16:
            return None                  # the mask rows are read in 16-byte pieces
        if dim != tc_attention.D or seq % (tc_attention.BQ * tc_attention.TILES) or M is not None:
            # head dim 32 or 64, S no multiple of 256, or an explicit mask: the default schedule only
            # (the other forms are built for head dim 128, whole 256-row query chunks and no mask)
            options = {k: v for k, v in options.items()
                       if k not in ("attn_persistent", "attn_kv128", "attn_overlap")}
        if M is not None:
            # the cubic exp2 variants clamp at 2^-120 instead of reaching 0, so a fully masked row
            # would sum to a tiny positive number instead of 0 (and end as 0, not NaN): MUFU only
            options = {k: v for k, v in options.items() if k not in ("attn_poly", "attn_pair_poly")}
        precise = bool(options.get("attn_precise", True))
        half = bool(options.get("attn_half", True)) and precise
        name = node.op.name
        kw = dict(names=(Q.name, K.name, V.name, O.name), prefix=prefix, precise=precise,
                  trace=bool(options.get("attn_trace", False)), half=half,
                  poly_every=int(options.get("attn_poly", tc_attention.POLY_EVERY)),
                  pingpong=bool(options.get("attn_pingpong", True)),
                  f16_int=int(options.get("attn_f16_int", 0)),
                  pack_after_turn=bool(options.get("attn_pack_after_turn", False)),
                  defer_sum=bool(options.get("attn_defer_sum", False)),
                  prefetch_next=int(options.get("attn_prefetch_next", 0)),
                  pack_in_turn=bool(options.get("attn_pack_in_turn", False)),
                  pair_poly=int(options.get("attn_pair_poly", 0)), dim=dim,
                  mask_name=M.name if M is not None else None)
        if options.get("attn_kv128", False):
            # 128-row key/value blocks: QK^T bound by the tensor core instead of shared memory
            from .kernels import tc_attention_kv128 as t128, vconv
            scratch = (f"{prefix}{name}__v16", f"{prefix}{name}__vflag")
            att = t128.attention_kv128_entry(name, bt, hd, seq, causal, scale,
                                             names=(Q.name, K.name, V.name, O.name), prefix=prefix,
                                             half=half, pingpong=bool(options.get("attn_pingpong", True)),
                                             ordered=bool(options.get("attn_ordered", False)),
                                             pack_in_turn=bool(options.get("attn_pack_in_turn", False)),
                                             scratch_names=scratch if half else None)
            if not half:
                return att
            return [vconv.vconv_entry(f"{name}_vconv", bt, hd, seq, names=(V.name,) + scratch,
                                      block_rows=t128.BKV), att]
        if options.get("attn_persistent", False):
            # opt-in persistent schedule (one CTA per SM, alternating row halves; see the module)
            from .kernels import tc_attention_persistent as tap, vconv
            scratch = (f"{prefix}{name}__v16", f"{prefix}{name}__vflag")
            att = tap.persistent_attention_entry(name, bt, hd, seq, causal, scale,
                                                 names=(Q.name, K.name, V.name, O.name), prefix=prefix,
                                                 half=half, ctas=int(options.get("sms", 148)),
                                                 scratch_names=scratch if half else None)
            if not half:
                return att
            return [vconv.vconv_entry(f"{name}_vconv", bt, hd, seq, names=(V.name,) + scratch), att]
        if not half:
            return tc_attention.attention_entry(name, bt, hd, seq, causal, scale, **kw)
        from .kernels import vconv
        scratch = (f"{prefix}{name}__v16", f"{prefix}{name}__vflag")
        pairs = bt * hd
        # opt-in: measured no faster on B200 (the co-running pre-pass takes the SM resources the
        # attention is bound by), kept for the runtime's two-stream schedule it exercises
        head = pairs // int(options.get("attn_overlap_split", 8)) if options.get("attn_overlap", False) else 0
        if head < 1 or head >= pairs:
            attn = tc_attention.attention_entry(name, bt, hd, seq, causal, scale, scratch_names=scratch, **kw)
            pre = vconv.vconv_entry(f"{name}_vconv", bt, hd, seq, names=(V.name,) + scratch, dim=dim)
            return [pre, attn]
        # The value pre-pass of all but the first `head` (batch, head) pairs runs on a side stream while
        # the attention of those first pairs runs: the pre-pass is bound by HBM bandwidth, which the
        # attention barely uses, and its CTAs fit beside the attention's (one per SM).  Only the first
        # group's pre-pass stays in the open.
        pre0 = vconv.vconv_entry(f"{name}_vconv", bt, hd, seq, names=(V.name,) + scratch, bh_range=(0, head))
        att0 = tc_attention.attention_entry(f"{name}_part0", bt, hd, seq, causal, scale, scratch_names=scratch,
                                            bh_range=(0, head), **kw)
        pre1 = vconv.vconv_entry(f"{name}_vconv1", bt, hd, seq, names=(V.name,) + scratch,
                                 bh_range=(head, pairs - head), ctas=int(options.get("attn_overlap_ctas", 148)))
        pre1["stream"] = 1
        pre1["after"] = [f"{name}_vconv"]
        pre1["carveout"] = 100          # the attention's shared-memory split, so the two can share an SM
        att1 = tc_attention.attention_entry(name, bt, hd, seq, causal, scale, scratch_names=scratch,
                                            bh_range=(head, pairs - head), **kw)
        att1["after"] = [f"{name}_vconv1"]
        att0["carveout"] = att1["carveout"] = 100
        return [pre0, att0, pre1, att1]
    return None
