"""Model plumbing on the host (mini_tensorrt_b200.executor): the int8-safe JSON
loader, the MatMul -> MatMulQ rewrite, the MatMulQ epilogue fusion and the arena
planner. No GPU needed."""
import json
import os

import numpy as np
import pytest

import oracle
from mini_tensorrt_b200 import executor as ex
from mini_tensorrt_b200.registry import GraphError, Node


def mlp_model(M=3, D=64, F=96, seed=0, residual=True):
    """x -> LayerNorm -> MatMul W1 -> Add b1 -> GeluTanh -> MatMul W2 -> Add b2 (-> Add x)."""
    rng = np.random.default_rng(seed)
    g = ex.Graph()
    T = lambda name, dt, shape, kind: g.add_tensor(ex.TensorInfo(name, dt, tuple(shape), kind))
    x = T("x", "f32", (M, D), "input")
    lg, lb = T("ln.g", "f32", (D,), "weight"), T("ln.b", "f32", (D,), "weight")
    w1, b1 = T("fc.w", "f32", (D, F), "weight"), T("fc.b", "f32", (F,), "weight")
    w2, b2 = T("proj.w", "f32", (F, D), "weight"), T("proj.b", "f32", (D,), "weight")
    h, t0, t1, t2, t3, t4 = (T(n, "f32", s, "intermediate") for n, s in
                             [("h", (M, D)), ("t0", (M, F)), ("t1", (M, F)), ("t2", (M, F)), ("t3", (M, D)),
                              ("t4", (M, D))])
    y = T("y", "f32", (M, D), "output")
    g.nodes = [Node("LayerNorm", [x, lg, lb], [h], {"eps": 1e-5}),
               Node("MatMul", [h, w1], [t0]), Node("Add", [t0, b1], [t1]), Node("GeluTanh", [t1], [t2]),
               Node("MatMul", [t2, w2], [t3])]
    if residual:
        g.nodes += [Node("Add", [t3, b2], [t4]), Node("Add", [x, t4], [y])]
    else:
        g.tensors[t4] = ex.TensorInfo("t4", "f32", (M, D), "intermediate")
        g.nodes += [Node("Add", [t3, b2], [y])]
    g.inputs, g.outputs = [x], [y]
    f32 = lambda *s, sc=1.0: (rng.standard_normal(s) * sc).astype(np.float32)
    weights = {lg: 1.0 + f32(D, sc=0.1), lb: f32(D, sc=0.1), w1: f32(D, F, sc=0.02), b1: f32(F, sc=0.02),
               w2: f32(F, D, sc=0.02), b2: f32(D, sc=0.02)}
    return ex.LoadedModel(g, weights)


def block_chain(n_blocks=2, M=3, D=64, F=96, seed=0):
    """n pre-LN MLP blocks whose output projection has no bias, so each block's
    residual Add folds into its second MatMulQ:
      x_{i+1} = x_i + MatMul(GeluTanh(MatMul(LayerNorm(x_i), W1) + b1), W2).
    From the second block on, the residual x_i is an intermediate in the arena,
    read by the fused MatMulQ's epilogue only."""
    rng = np.random.default_rng(seed)
    g = ex.Graph()
    T = lambda name, dt, shape, kind: g.add_tensor(ex.TensorInfo(name, dt, tuple(shape), kind))
    f32 = lambda *s, sc=1.0: (rng.standard_normal(s) * sc).astype(np.float32)
    x = T("x", "f32", (M, D), "input")
    g.inputs = [x]
    weights = {}
    cur = x
    for i in range(n_blocks):
        lg, lb = T(f"b{i}.ln.g", "f32", (D,), "weight"), T(f"b{i}.ln.b", "f32", (D,), "weight")
        w1, b1 = T(f"b{i}.fc.w", "f32", (D, F), "weight"), T(f"b{i}.fc.b", "f32", (F,), "weight")
        w2 = T(f"b{i}.proj.w", "f32", (F, D), "weight")
        weights.update({lg: 1.0 + f32(D, sc=0.1), lb: f32(D, sc=0.1), w1: f32(D, F, sc=0.02),
                        b1: f32(F, sc=0.02), w2: f32(F, D, sc=0.02)})
        h, t0, t1, t2, t3 = (T(f"b{i}.{n}", "f32", s, "intermediate") for n, s in
                             [("h", (M, D)), ("t0", (M, F)), ("t1", (M, F)), ("t2", (M, F)), ("t3", (M, D))])
        last = i == n_blocks - 1
        nxt = T("y" if last else f"x{i + 1}", "f32", (M, D), "output" if last else "intermediate")
        g.nodes += [Node("LayerNorm", [cur, lg, lb], [h], {"eps": 1e-5}),
                    Node("MatMul", [h, w1], [t0]), Node("Add", [t0, b1], [t1]), Node("GeluTanh", [t1], [t2]),
                    Node("MatMul", [t2, w2], [t3]), Node("Add", [cur, t3], [nxt])]
        cur = nxt
    g.outputs = [cur]
    return ex.LoadedModel(g, weights)


def _independent_intervals(g):
    """Live intervals computed here from first principles (not by the planner):
    an intermediate is live from its producer's step to the step of its last
    reader, where a fused MatMulQ also reads the tensors its bias and residual
    attributes name."""
    order = g.topo_order()
    live = {}
    for step, ni in enumerate(order):
        nd = g.nodes[ni]
        for t in nd.outputs:
            if g.tensors[t].kind == "intermediate":
                live.setdefault(t, [step, step])
        reads = list(nd.inputs) + [nd.attrs[k] for k in ("bias", "residual") if k in nd.attrs]
        for t in reads:
            if t in live:
                live[t][1] = step
    return live


def test_json_round_trip_keeps_every_dtype(tmp_path):
    m = mlp_model()
    g = m.graph
    q = g.add_tensor(ex.TensorInfo("q", "i8", (4, 5), "weight"))
    ids = g.add_tensor(ex.TensorInfo("ids", "i32", (3,), "weight"))
    m.weights[q] = np.arange(-10, 10, dtype=np.int8).reshape(4, 5)
    m.weights[ids] = np.array([7, -1, 2 ** 30], dtype=np.int32)
    path = str(tmp_path / "model.json")
    ex.save_json_model(m, path)
    back = ex.load_json_model(path)
    assert [t for t in back.graph.tensors] == [t for t in g.tensors]
    assert [(n.op_type, n.inputs, n.outputs, n.attrs) for n in back.graph.nodes] == \
        [(n.op_type, n.inputs, n.outputs, n.attrs) for n in g.nodes]
    for tid, w in m.weights.items():
        assert back.weights[tid].dtype == w.dtype and np.array_equal(back.weights[tid], w)


@pytest.mark.parametrize("edit,msg", [
    (lambda j: j["tensors"][0].update(dtype="f16"), "unsupported dtype"),
    (lambda j: j["tensors"][0].update(kind="scratch"), "unknown tensor kind"),
    (lambda j: j["tensors"].append(dict(j["tensors"][0])), "duplicate tensor name"),
    (lambda j: j["tensors"][1].update(offset=10 ** 9), "exceeds weights blob"),
    (lambda j: j["tensors"][1].update(nbytes=4), "byte size mismatch"),
    (lambda j: j["nodes"][0]["inputs"].__setitem__(0, "nope"), "unknown tensor"),
])
def test_loader_errors(tmp_path, edit, msg):
    """The reference loader's errors (src/frontend/json/json_loader.cpp:17-31, 78-127)."""
    path = str(tmp_path / "model.json")
    ex.save_json_model(mlp_model(), path)
    with open(path) as f:
        j = json.load(f)
    edit(j)
    with open(path, "w") as f:
        json.dump(j, f)
    with pytest.raises(GraphError, match=msg):
        ex.load_json_model(path)


def test_topo_order_rules():
    g = mlp_model().graph
    order = g.topo_order()
    pos = {ni: i for i, ni in enumerate(order)}
    prod = {t: ni for ni, n in enumerate(g.nodes) for t in n.outputs}
    for ni, n in enumerate(g.nodes):
        for t in n.inputs:
            if t in prod:
                assert pos[prod[t]] < pos[ni]
    g2 = mlp_model().graph
    g2.nodes.append(Node("GeluTanh", [g2.nodes[0].inputs[0]], [g2.nodes[0].outputs[0]]))
    with pytest.raises(GraphError, match="more than one producer"):
        g2.topo_order()
    g3 = mlp_model().graph
    g3.nodes[0].inputs[0] = g3.nodes[-1].outputs[0]  # LayerNorm reads y: a cycle
    g3.tensors[g3.nodes[-1].outputs[0]] = ex.TensorInfo("y", "f32", (3, 64), "intermediate")
    with pytest.raises(GraphError, match="cycle"):
        g3.topo_order()


def test_quantize_rewrites_matmul_with_the_reference_packer():
    m = mlp_model()
    q = ex.quantize_matmuls(m)
    ops = [n.op_type for n in q.graph.nodes]
    assert ops.count("MatMulQ") == 2 and "MatMul" not in ops
    for n in q.graph.nodes:
        if n.op_type != "MatMulQ":
            continue
        x, wq, sc = n.inputs
        src = next(t for t in range(len(m.graph.tensors)) if m.graph.tensors[t].name + ".q8" ==
                   q.graph.tensors[wq].name)
        qo, so = oracle.quantize_per_channel(m.weights[src])  # the reference packer, restated
        assert q.graph.tensors[wq].dtype == "i8" and np.array_equal(q.weights[wq], qo)
        assert np.array_equal(q.weights[sc].view(np.uint32), so.view(np.uint32))
        assert src not in q.weights  # the fp32 weight is no longer needed


def test_fusion_patterns():
    q = ex.quantize_matmuls(mlp_model(residual=True))
    f = ex.fuse_matmulq_epilogues(q)
    ops = [(n.op_type, n.attrs.get("epilogue"), "bias" in n.attrs) for n in f.graph.nodes]
    # LN, MatMulQ{bias, gelu}, MatMulQ{bias}, Add(x, t4)
    assert ops == [("LayerNorm", None, False), ("MatMulQ", "gelu", True), ("MatMulQ", None, True),
                   ("Add", None, False)]
    # without the bias Add the residual folds into the second MatMulQ
    g = q.graph
    mm2 = next(n for n in g.nodes if n.op_type == "MatMulQ" and n.inputs[0] != g.nodes[0].outputs[0])
    t3 = mm2.outputs[0]
    add_b = next(n for n in g.nodes if n.op_type == "Add" and n.inputs[0] == t3)
    g.nodes.remove(add_b)
    last = next(n for n in g.nodes if n.op_type == "Add" and n.inputs[0] == g.inputs[0])
    last.inputs[1] = t3
    f2 = ex.fuse_matmulq_epilogues(q)
    assert [(n.op_type, n.attrs.get("epilogue")) for n in f2.graph.nodes][-1] == ("MatMulQ", "residual")
    # a MatMulQ output read twice is not fused
    q3 = ex.quantize_matmuls(mlp_model())
    g3 = q3.graph
    t0 = g3.nodes[1].outputs[0]
    g3.outputs.append(t0)
    f3 = ex.fuse_matmulq_epilogues(q3)
    assert not any(n.attrs.get("epilogue") == "gelu" for n in f3.graph.nodes)


def test_plan_memory_aligns_and_never_overlaps_live_tensors():
    for seed in range(4):
        m = ex.fuse_matmulq_epilogues(ex.quantize_matmuls(mlp_model(M=1 + seed, seed=seed)))
        g = m.graph
        plan = ex.plan_memory(g)
        ivs = {t: (a, b, nb) for t, a, b, nb in plan.intervals}
        for t, off in plan.offset.items():
            assert off % ex.ARENA_ALIGNMENT == 0
            assert off + g.tensors[t].nbytes <= plan.total_bytes
        for t, (a, b, nb) in ivs.items():
            for u, (c, d, nu) in ivs.items():
                if t < u and a <= d and c <= b:  # live at the same time
                    o1, o2 = plan.offset[t], plan.offset[u]
                    assert o1 + nb <= o2 or o2 + nu <= o1
        assert plan.total_bytes % ex.ARENA_ALIGNMENT == 0
        assert plan.total_bytes <= sum(-(-nb // 256) * 256 for _, _, nb in ivs.values())


def test_reference_fused_node_becomes_matmulq_with_epilogue():
    """A graph the reference's fuse_matmul_bias_gelu already rewrote."""
    m = mlp_model()
    g = m.graph
    mm, add, gelu = g.nodes[1], g.nodes[2], g.nodes[3]
    g.nodes[1:4] = [Node("FusedMatMulBiasGeluTanh", [mm.inputs[0], mm.inputs[1], add.inputs[1]],
                         list(gelu.outputs))]
    q = ex.quantize_matmuls(m)
    n = q.graph.nodes[1]
    assert n.op_type == "MatMulQ" and n.attrs == {"bias": add.inputs[1], "epilogue": "gelu"}
    assert n.outputs == gelu.outputs
    # the executor's node checks accept it (no device needed for the planner)
    assert ex.plan_memory(q.graph).total_bytes > 0


def test_epilogue_operands_stay_live_until_their_reader():
    """A residual that is an intermediate and read only by a fused MatMulQ's
    epilogue must not share arena bytes with anything written before that MatMulQ
    runs (here: the first MatMulQ's output of the same block)."""
    m = ex.fuse_matmulq_epilogues(ex.quantize_matmuls(block_chain(n_blocks=3, M=2)))
    g = m.graph
    fused = [n for n in g.nodes if n.op_type == "MatMulQ" and n.attrs.get("epilogue") == "residual"]
    assert len(fused) == 3
    assert any(g.tensors[n.attrs["residual"]].kind == "intermediate" for n in fused)
    plan = ex.plan_memory(g)
    live = _independent_intervals(g)
    assert set(live) == set(plan.offset)
    for t, (a, b) in live.items():
        for u, (c, d) in live.items():
            if t < u and a <= d and c <= b:
                o1, o2 = plan.offset[t], plan.offset[u]
                assert o1 + g.tensors[t].nbytes <= o2 or o2 + g.tensors[u].nbytes <= o1, \
                    (g.tensors[t].name, g.tensors[u].name)


def test_epilogue_operand_orders_its_producer_first():
    """A node whose bias or residual is produced by a node listed later is ordered
    after that producer, and the producer's output counts as read (not single-use
    when something else reads it too)."""
    g = ex.Graph()
    T = lambda name, shape, kind: g.add_tensor(ex.TensorInfo(name, "f32", tuple(shape), kind))
    x, wq, sc = T("x", (2, 4), "input"), T("wq", (4, 4), "weight"), T("sc", (4,), "weight")
    r, y = T("r", (2, 4), "intermediate"), T("y", (2, 4), "output")
    g.tensors[wq] = ex.TensorInfo("wq", "i8", (4, 4), "weight")
    g.nodes = [Node("MatMulQ", [x, wq, sc], [y], {"epilogue": "residual", "residual": r}),
               Node("GeluTanh", [x], [r])]
    g.inputs, g.outputs = [x], [y]
    assert g.topo_order() == [1, 0]
    assert ex.node_reads(g.nodes[0]) == [x, wq, sc, r]
