"""CPU tests of the C++ front end: graph building, autograd, the scheduler's
materialisation rules and the CUDA C renderer (no GPU needed -- buffers stay
unallocated, rendered kernels are compiled with NVRTC for sm_100a but not
run).  Scheduler cases mirror the reference's own tests in
src/schedule.rs:367-571 and src/tensor.rs:1128-1314."""
import ctypes
import ctypes.util

import numpy as np
import pytest

from ferrograd_b200 import front as F

U = F.UOp


def buffer_ids(item):
    return [v for k, v in item["inputs"] if k == "buffer"]


# ----------------------------------------------------------------- scheduler
def test_nested_reductions_materialize_via_shared_buffer_handles():
    inp = U.buffer([2, 2])
    inner = U.reduce(inp, "add", [1])
    outer = U.reduce(inner, "add", [0])
    items = F.schedule_uops([outer])
    assert len(items) == 2
    assert items[1]["inputs"][0] == ("buffer", items[0]["output"])


def test_shared_subexpression_materializes_once():
    left, right = U.buffer([2, 2]), U.buffer([2, 2])
    shared = U.add(left, right)
    s = U.reduce(shared, "add", [1])
    m = U.reduce(shared, "max", [1])
    items = F.schedule_uops([U.add(s, m)])
    assert len(items) == 4
    assert items[1]["inputs"][0] == ("buffer", items[0]["output"])
    assert items[2]["inputs"][0] == ("buffer", items[0]["output"])
    assert items[3]["inputs"] == [("buffer", items[1]["output"]), ("buffer", items[2]["output"])]


def test_parameterize_gives_each_shrink_occurrence_its_own_scalar_input():
    inp = U.buffer([3, 2])
    zero = U.const_int(0)
    left = U.shrink(inp, [zero, zero], [2, 2])
    right = U.shrink(U.reshape(inp, [3, 2]), [zero, zero], [2, 2])
    items = F.schedule_uops([U.add(left, right)])
    scalars = [i for it in items for i in it["inputs"] if i[0] != "buffer"]
    assert len(scalars) == 2


def test_parameterize_store_turns_shrink_start_into_scalar_input():
    src, dst = U.buffer([3, 2]), U.buffer([2, 2])
    narrowed = U.shrink(src, [U.const_int(1), U.const_int(0)], [2, 2])
    items = F.schedule_uops([U.after(dst, U.store(dst, narrowed))])
    assert len(items) == 1 and items[0]["kind"] == "store"
    ins = items[0]["inputs"]
    assert ins[0][0] == "buffer" and ins[1][0] == "buffer" and ins[2] == ("i32", 1)
    assert ins[0][1] == dst.buffer_id()


def test_shared_movement_view_does_not_materialize():
    left, right = U.buffer([2, 2]), U.buffer([2, 2])
    moved = U.reshape(U.add(left, right), [2, 2])
    s = U.reduce(moved, "add", [1])
    m = U.reduce(moved, "max", [1])
    items = F.schedule_uops([U.add(s, m)])
    assert len(items) == 3
    assert [k for k, _ in items[0]["inputs"]] == ["buffer", "buffer"]
    assert [k for k, _ in items[1]["inputs"]] == ["buffer", "buffer"]
    assert items[2]["inputs"] == [("buffer", items[0]["output"]), ("buffer", items[1]["output"])]


def test_shared_movement_view_stays_inlined_for_assignments():
    left, right = U.buffer([2, 2]), U.buffer([2, 2])
    dst_a, dst_b = U.buffer([2, 2]), U.buffer([2, 2])
    moved = U.permute(U.add(left, right), [1, 0])
    plan = F.schedule_uops([U.after(dst_a, U.store(dst_a, moved)),
                            U.after(dst_b, U.store(dst_b, moved))])
    assert len(plan) == 2
    assert all(it["kind"] == "store" and it["output"] is None for it in plan)
    assert all(len(it["inputs"]) == 3 for it in plan)


def test_interning_makes_equal_graphs_identical():
    a = U.buffer([4])
    assert U.add(a, a).same(U.add(a, a))
    assert not U.add(a, a).same(U.mul(a, a))


def test_interner_holds_live_nodes_only():
    """The interning table grows past its initial size, finds every live node
    again (also after entries around it were deleted), and a node leaves it
    when the node dies."""
    base = F.interner_size()
    a = U.buffer([4])
    nodes = [U.add(a, U.const_int(i)) for i in range(5000)]
    grown = F.interner_size()
    assert grown >= base + 2 * 5000  # each sum and its literal
    # drop every other node: their deletions shift the probe runs of the rest
    kept = nodes[1::2]
    del nodes
    assert F.interner_size() <= grown - 2 * 2500
    found = all(n.same(U.add(a, U.const_int(2 * j + 1))) for j, n in enumerate(kept))
    other = kept[0].same(U.add(a, U.const_int(0)))
    assert found and not other
    del kept
    assert F.interner_size() == base + 2  # a: its buffer and reshape


# --------------------------------------------------------------- tensor API
def test_add_is_lazy_and_shapes_infer():
    a = F.tensor([1.0, 2.0])
    b = F.tensor([3.0, 4.0])
    c = a.add(b)
    assert not c.is_realized() and a.is_realized()
    assert c.shape == (2,)
    x = F.Tensor.empty([4, 3])
    assert x.permute([1, 0]).shape == (3, 4)
    assert x.sum([0]).shape == (1, 3)
    assert x.narrow(0, 1, 2).shape == (2, 3)
    assert x.matmul(F.Tensor.empty([3, 5])).shape == (4, 5)
    assert x.add(F.Tensor.empty([3])).shape == (4, 3)


def test_dtypes_follow_tensor_new():
    assert F.tensor(np.array([1, 2, 3], np.int32)).dtype == "i32"
    assert F.tensor(np.array([True, False])).dtype == "bool"
    assert F.tensor([1.5]).dtype == "f32"
    z = F.Tensor.zeros([2])
    assert z.relu().dtype == "f32"


@pytest.mark.parametrize("fn,msg", [
    (lambda: F.Tensor.empty([2, 3]).add(F.Tensor.empty([4, 3])), "broadcast"),
    (lambda: F.Tensor.empty([2, 3]).reshape([4]), "reshape: numel mismatch"),
    (lambda: F.Tensor.empty([2, 3]).permute([0, 0]), "duplicated"),
    (lambda: F.Tensor.empty([2, 3]).narrow(1, 2, 2), "out of bounds"),
    (lambda: F.Tensor.empty([2, 3]).matmul(F.Tensor.empty([2, 3])), "inner dim mismatch"),
    (lambda: F.Tensor.empty([2, 3]).sum([2]), "out of range"),
    (lambda: F.Tensor.empty([2, 3]).backward(), "scalar loss"),
    (lambda: F.Tensor.empty([2]).assign(F.Tensor.empty([3])), "assign: shape mismatch"),
    (lambda: F.Tensor.empty([2]).add(F.Tensor.empty([2])).assign(F.Tensor.empty([2])),
     "buffer identity"),
    (lambda: F.Sgd([], 0.1), "at least one parameter"),
])
def test_misuse_panics_like_the_reference(fn, msg):
    with pytest.raises(RuntimeError, match=msg):
        fn()


def test_sgd_step_requires_gradients():
    p = F.Tensor.empty([2]).with_requires_grad(True)
    with pytest.raises(RuntimeError, match="requires parameter gradients"):
        F.Sgd([p], 0.1).step()


def test_sgd_dedupes_shared_parameters():
    p = F.Tensor.empty([2]).with_requires_grad(True)
    assert len(F.Sgd([p, p], 0.1).params) == 1


def test_backward_targets_live_tensors_that_require_grad():
    x = F.Tensor.empty([3]).with_requires_grad(True)
    y = F.Tensor.empty([3]).with_requires_grad(True)
    z = F.Tensor.empty([3])
    loss = x.mul(y).add(z).sum([0])
    loss.backward()
    assert x.grad() is not None and y.grad() is not None
    assert z.grad() is None
    assert not x.grad().requires_grad()
    loss.backward()  # accumulates: grad = old + new
    assert "Add" in x.grad()._graph().splitlines()[-1]


def test_gradient_of_an_axis_expanded_to_zero_keeps_the_source_shape():
    """An axis of 1 expanded to 0 gets the sum over nothing as its gradient:
    reduced back to 1, never a 0-element gradient viewed as the source's
    shape (which would read past the end of the buffer)."""
    x = F.Tensor.empty([1, 64]).with_requires_grad(True)
    loss = x.expand([0, 64]).relu().sum([0, 1])
    loss.backward()
    g = x.grad()
    assert g.shape == (1, 64)
    assert "ReduceAxis" in g._graph()


def test_cross_entropy_of_empty_logits_keeps_the_reference_graph(monkeypatch):
    """The fused cross-entropy kernel rejects empty logits, so the default
    mode builds the reference's decomposed graph for them."""
    monkeypatch.delenv("FG_FRONT_EXACT", raising=False)
    t = F.Tensor.zeros([0, 10])
    assert "XentLoss" not in F.Tensor.empty([0, 10]).cross_entropy(t)._graph()
    assert "XentLoss" in F.Tensor.empty([4, 10]).cross_entropy(F.Tensor.zeros([4, 10]))._graph()


def test_internal_reshape_keeps_the_element_count():
    with pytest.raises(RuntimeError, match="numel mismatch"):
        U.reshape(U.buffer([4]), [3])


def test_gradient_of_untracked_target_is_zeros():
    x = F.Tensor.empty([2, 2])
    w = F.Tensor.empty([2, 1]).with_requires_grad(True)
    loss = x.matmul(w).sum([0, 1])
    gx, gw = loss.gradient([x, w])
    assert gx.shape == (2, 2) and gw.shape == (2, 1)
    assert "Const" in gx._graph() and "Buffer" not in gx._graph()


def test_linear_init_is_the_reference_kaiming_stream():
    F.reset_init_seed(42)
    layer = F.Linear(4, 5)
    assert layer.weight.shape == (5, 4) and layer.bias.shape == (5,)
    assert layer.weight.requires_grad() and layer.bias.requires_grad()
    seed_after = F.init_seed()
    F.reset_init_seed(42)
    F.Linear.without_bias(4, 5)
    assert F.init_seed() == seed_after  # 20 draws either way
    assert len(F.Linear(3, 2).parameters()) == 2


# ----------------------------------------------------------- the MLP step
def build_step(dims, batch, lr=0.01, empty_inputs=False):
    F.reset_init_seed(42)
    model = F.Mlp(dims)
    if empty_inputs:
        x, t = F.Tensor.empty([batch, dims[0]]), F.Tensor.empty([batch, dims[-1]])
    else:
        rng = np.random.default_rng(0)
        x = F.tensor(rng.random((batch, dims[0]), np.float32))
        t = F.one_hot(np.arange(batch) % dims[-1], dims[-1])
    loss = model(x).cross_entropy(t)
    loss.backward()
    ps = model.parameters()
    for p in ps:  # Sgd::step's graph, scheduled without running
        p.assign(p.detach().sub(p.grad().mul(F.Tensor.scalar(lr))))
    return model, ps, loss


def test_mlp_step_schedule_config1_exact_mode_is_the_references(monkeypatch):
    """Exact mode schedules the reference's kernels: 23 for the config-1
    step, cross_entropy decomposed as src/tensor.rs:715-752 builds it."""
    monkeypatch.setenv("FG_FRONT_EXACT", "1")
    _, ps, _ = build_step((784, 128, 10), 256)
    items = F.schedule(ps)
    stores = [it for it in items if it["kind"] == "store"]
    assert len(stores) == 4  # one in-place update per parameter
    assert len(items) == 23
    assert all(it["route"] == "rendered" for it in items)


def test_mlp_step_schedule_config1(monkeypatch):
    """Default mode: cross_entropy is one fused op whose gradient pass is a
    kernel of its own (the decomposed graph's 9 kernels become 1), the
    logits it reads are materialised, matmul's contiguous() copies of the
    (already contiguous) weights are read in place (2 kernels fewer), each
    Linear's contraction stays in its bias-add kernel (2 fewer), and ReLU's
    mask is recomputed from z by its consumers, the masked gradient keeping
    its dX contraction (2 fewer)."""
    monkeypatch.delenv("FG_FRONT_EXACT", raising=False)
    _, ps, loss = build_step((784, 128, 10), 256)
    items = F.schedule(ps)
    stores = [it for it in items if it["kind"] == "store"]
    assert len(stores) == 4  # one in-place update per parameter
    assert len(items) == 8
    routes = [it["route"] for it in items]
    assert routes.count("xent") == 1
    assert any(st.endswith("+bias") for it in items for st in it["steps"])
    assert F.schedule([loss])[-1]["route"] == "xent"
    # The layer-1 forward contraction and the fused dW1 -> SGD store go to
    # the tensor cores; the 10-wide layer is too small and is rendered.
    assert routes.count("gemm") == 1
    assert any(it["steps"] == ["gemm 128x784x256"] for it in stores)


def test_mlp_step_schedule_config5_routes_contractions_to_gemm(monkeypatch):
    monkeypatch.delenv("FG_FRONT_EXACT", raising=False)
    _, ps, _ = build_step((4096, 4096, 4096, 10), 8192, empty_inputs=True)
    items = F.schedule(ps)
    steps = [s for it in items for s in it["steps"]]
    gemms = sorted(s for s in steps if s.startswith("gemm"))
    # 3 forward, 3 dW and 1 dX contraction at config-5 size; the 10-class
    # layer's dX (K = 10) is rendered
    assert len(gemms) == 7, gemms
    # fwd 1 and fwd 2 with the bias epilogue, dX 2 plain
    assert gemms.count("gemm 8192x4096x4096 +bias") == 2, gemms
    assert gemms.count("gemm 8192x4096x4096") == 1
    assert gemms.count("gemm 4096x4096x8192") == 2  # dW 1, dW 2
    assert {"gemm 8192x10x4096 +bias", "gemm 10x4096x8192"} <= set(gemms)
    assert "gemm 8192x4096x10" not in gemms
    assert "reduce_cols" in steps  # bias gradients


# ------------------------------------------------------------------ renderer
def nvrtc():
    name = ctypes.util.find_library("nvrtc") or "libnvrtc.so.12"
    try:
        return ctypes.CDLL(name)
    except OSError:
        for cand in ("/usr/local/cuda/lib64/libnvrtc.so", "libnvrtc.so.12"):
            try:
                return ctypes.CDLL(cand)
            except OSError:
                pass
    pytest.skip("libnvrtc not found")


def nvrtc_compile(lib, src):
    prog = ctypes.c_void_p()
    assert lib.nvrtcCreateProgram(ctypes.byref(prog), src.encode(), b"k.cu", 0, None, None) == 0
    opts = [b"-arch=sm_100a", b"--std=c++17", b"-default-device"]
    rc = lib.nvrtcCompileProgram(prog, len(opts), (ctypes.c_char_p * len(opts))(*opts))
    n = ctypes.c_size_t()
    lib.nvrtcGetProgramLogSize(prog, ctypes.byref(n))
    log = ctypes.create_string_buffer(max(1, n.value))
    lib.nvrtcGetProgramLog(prog, log)
    lib.nvrtcDestroyProgram(ctypes.byref(prog))
    return rc, log.value.decode(errors="replace")


@pytest.mark.parametrize("exact", ["1", "0"])
def test_every_rendered_kernel_of_the_step_compiles_for_sm100a(monkeypatch, exact):
    monkeypatch.setenv("FG_FRONT_EXACT", exact)
    lib = nvrtc()
    _, ps, loss = build_step((784, 128, 10), 256)
    items = F.schedule(ps, with_source=True) + F.schedule([loss], with_source=True)
    seen = set()
    for it in items:
        if it["source"] in seen:
            continue
        seen.add(it["source"])
        rc, log = nvrtc_compile(lib, it["source"])
        assert rc == 0, log + "\n" + it["source"]
    assert len(seen) > (10 if exact == "1" else 5)


def test_rendered_reduction_order_and_rounding():
    x = F.Tensor.empty([3, 8])
    src = F.schedule([x.sum([1])], with_source=True)[0]["source"]
    # R = 8: two blocks of four lanes folded left to right into one accumulator.
    assert "< 2LL" in src and src.count("__fadd_rn") == 4
    y = F.Tensor.empty([3, 10])
    src = F.schedule([y.sum([1])], with_source=True)[0]["source"]
    assert "< 10LL" in src and src.count("__fadd_rn") == 1  # sequential
    m = F.schedule([y.max([1])], with_source=True)[0]["source"]
    assert "(-INFINITY)" in m and " > " in m
    e = F.schedule([x.exp2().log2().sqrt().reciprocal()], with_source=True)[0]["source"]
    assert "exp2((double)" in e and "log2((double)" in e
    assert "__fsqrt_rn" in e and "__frcp_rn" in e
    assert "fma" not in e


def test_const_folding_follows_symbolic_simple():
    x = F.Tensor.empty([4]).with_requires_grad(True)
    loss = x.sum([0])
    (g,) = loss.gradient([x])
    # The gradient is expand(full(1.0)) -- a constant kernel: no loads.
    src = F.schedule([g], with_source=True)[0]["source"]
    assert "1.0f" in src and "p1[" not in src


def test_reduction_over_an_empty_axis_reads_nothing():
    """sum/max over a zero-length axis is the identity (0 / -inf); the
    rendered kernel must not load from the empty buffer."""
    z = F.Tensor.empty([0, 3])
    for red, ident in ((z.sum([0]), "0.0f"), (z.max([0]), "(-INFINITY)")):
        src = F.schedule([red], with_source=True)[0]["source"]
        body = src.split("{", 1)[1]
        assert "p1[" not in body and ident in body


def test_only_zeros_tensors_render_as_known_zero():
    """Tensor::zeros buffers that nothing has written may be used as the
    value 0; uploaded data never is."""
    z = F.Tensor.zeros([4])
    d = F.tensor([1.0, 2.0, 3.0, 4.0])
    src = F.schedule([z.add(d)], with_source=True)[0]["source"]
    body = src.split("{", 1)[1]
    # only the data tensor is loaded (a scalar or a 128-bit load)
    assert "p1[" not in body and "p1 +" not in body
    assert "p2[" in body or "p2 +" in body


def test_opt_parsing_matches_the_reference():
    """parse_optimize_config (src/optimize/mod.rs:80-108) and its tests
    (src/optimize/mod.rs, mod tests): unset/empty/all enable every pass,
    0/off/none disable every pass, otherwise a comma list of pass names
    (unknown names ignored, whitespace trimmed)."""
    from ferrograd_b200 import front as F
    allp = {"symbolic": True, "upcast": True, "unroll": True}
    nonep = {"symbolic": False, "upcast": False, "unroll": False}
    for raw in ("", "all", "1", "on", "  all  "):
        assert F._front.parse_optimize_config(raw) == allp, raw
    for raw in ("0", "off", "none", " none "):
        assert F._front.parse_optimize_config(raw) == nonep, raw
    assert F._front.parse_optimize_config("symbolic") == {"symbolic": True, "upcast": False,
                                                          "unroll": False}
    assert F._front.parse_optimize_config("symbolic,upcast,unroll,unknown") == allp
    assert F._front.parse_optimize_config(" unroll , symbolic") == {"symbolic": True,
                                                                   "upcast": False,
                                                                   "unroll": True}


# -------------------------------------------------- thread mapping (default mode)
def test_elementwise_kernels_use_128_bit_accesses():
    """An elementwise chain over contiguous operands whose innermost extent is
    a multiple of 4 loads and stores 4 elements at a time (float4); a
    broadcast operand is read once per group, a strided one element-wise."""
    def data(*shape):  # uploaded data: never treated as known zeros
        return F.tensor(np.ones(shape, np.float32))
    a, b, bias = data(8, 16), data(8, 16), data(16)
    src = F.schedule([a.mul(b).add(bias.reshape([1, 16]).expand([8, 16]))],
                     with_source=True)[0]["source"]
    assert src.count("*reinterpret_cast<const float4 *>") == 2 * 3  # a, b, bias per group
    assert "make_float4" in src
    t = data(16, 8).permute([1, 0])  # innermost stride 16: gathered
    src = F.schedule([a.add(t)], with_source=True)[0]["source"]
    assert src.count("*reinterpret_cast<const float4 *>") == 2 and "p2[" in src
    odd = data(5, 3)  # innermost extent not a multiple of 4
    src = F.schedule([odd.add(odd)], with_source=True)[0]["source"]
    assert "float4" not in src


def test_long_reductions_use_warp_and_block_mappings(monkeypatch):
    monkeypatch.delenv("FG_FRONT_EXACT", raising=False)
    x = F.Tensor.empty([64, 100])
    rows = F.schedule([x.sum([1])], with_source=True)[0]["source"]
    assert "__shfl_xor_sync" in rows and "r < 100LL" not in rows
    cols = F.schedule([x.max([0])], with_source=True)[0]["source"]
    assert "__syncthreads" in cols and "fg_sm_f" in cols
    short = F.schedule([F.Tensor.empty([64, 8]).sum([1])], with_source=True)[0]["source"]
    assert "__shfl" not in short and "__syncthreads" not in short


def test_exact_mode_keeps_the_sequential_reduction_order(monkeypatch):
    monkeypatch.setenv("FG_FRONT_EXACT", "1")
    x = F.Tensor.empty([64, 100])
    for red in (x.sum([1]), x.max([0])):
        src = F.schedule([red], with_source=True)[0]["source"]
        assert "__shfl" not in src and "__syncthreads" not in src
