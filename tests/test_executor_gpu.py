"""DeviceExecutor (mini_tensorrt_b200.executor) on a GPT-2 MLP block loaded from
the reference's JSON format: quantized, fused and run on the device, against the
reference's ops restated on the CPU (oracle MatMulQ for every Linear)."""
import numpy as np
import pytest
import torch

import oracle
from mini_tensorrt_b200 import executor as ex
from mini_tensorrt_b200.registry import GraphError, Node
from tests.conftest import rel_err
from tests.test_executor_host import block_chain, mlp_model

pytestmark = pytest.mark.gpu


def _layernorm(x, g, b, eps):
    # the reference's LayerNorm (src/ops/kernels_transformer.cpp:40-52) in fp32
    mean = x.mean(axis=1, keepdims=True, dtype=np.float32)
    c = (x - mean).astype(np.float32)
    var = (c * c).mean(axis=1, keepdims=True, dtype=np.float32)
    return (c * (np.float32(1.0) / np.sqrt(var + np.float32(eps))) * g + b).astype(np.float32)


def _gelu_new(u):
    k = np.float32(0.7978845608028654)
    return (np.float32(0.5) * u * (np.float32(1.0) + np.tanh(k * (u + np.float32(0.044715) * u ** 3))))


def reference_forward(m, x):
    """The graph's meaning with the reference's ops: every MatMul of the fp32 graph as
    the reference MatMulQ on the packer's int8 weights."""
    g, W = m.graph, m.weights
    val = {g.inputs[0]: x}
    for ni in g.topo_order():
        n = g.nodes[ni]
        a = [val[i] if i in val else W[i] for i in n.inputs]
        if n.op_type == "LayerNorm":
            r = _layernorm(a[0], a[1], a[2], n.attrs["eps"])
        elif n.op_type == "MatMul":
            q, s = oracle.quantize_per_channel(a[1])
            r = oracle.matmul_q8(a[0], q, s)
        elif n.op_type == "Add":
            r = (a[0] + a[1]).astype(np.float32)
        elif n.op_type == "GeluTanh":
            r = _gelu_new(a[0]).astype(np.float32)
        val[n.outputs[0]] = r
    return val[g.outputs[0]]


@pytest.mark.parametrize("M", [1, 8, 64])
@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_mlp_block_from_json_matches_reference(cuda_device, tmp_path, M, mode):
    m = mlp_model(M=M, D=768, F=3072, seed=M)
    path = str(tmp_path / "mlp.json")
    ex.save_json_model(m, path)
    loaded = ex.load_json_model(path)
    run_model = ex.fuse_matmulq_epilogues(ex.quantize_matmuls(loaded))
    assert sum(n.op_type == "MatMulQ" for n in run_model.graph.nodes) == 2
    exe = ex.DeviceExecutor(run_model, cuda_device, mode=mode)
    x = np.random.default_rng(M).standard_normal((M, 768)).astype(np.float32)
    y = exe.run(x)[0]
    want = reference_forward(m, x)
    err = rel_err(y, want)
    assert err <= (1e-4 if mode == "fp32" else 2e-2), f"rel err {err:.3e}"


def test_run_allocates_no_device_memory(cuda_device):
    m = ex.fuse_matmulq_epilogues(ex.quantize_matmuls(mlp_model(M=4, D=768, F=3072)))
    exe = ex.DeviceExecutor(m, cuda_device, mode="bf16")
    x = np.random.default_rng(0).standard_normal((4, 768)).astype(np.float32)
    first = exe.run(x)[0]
    torch.cuda.synchronize()
    before = torch.cuda.memory_stats(cuda_device)["allocation.all.allocated"]
    for _ in range(3):
        again = exe.run(x)[0]
    torch.cuda.synchronize()
    assert torch.cuda.memory_stats(cuda_device)["allocation.all.allocated"] == before
    assert np.array_equal(first, again)


def test_unsupported_ops_fail_at_setup(cuda_device):
    m = ex.quantize_matmuls(mlp_model(M=2, D=64, F=96))
    m.graph.nodes[3] = Node("Gelu", list(m.graph.nodes[3].inputs), list(m.graph.nodes[3].outputs))
    with pytest.raises(GraphError, match="unsupported op 'Gelu'"):
        ex.DeviceExecutor(ex.fuse_matmulq_epilogues(m), cuda_device)
    # a broadcast Add that does not follow a MatMulQ has no device kernel
    m2 = ex.quantize_matmuls(mlp_model(M=2, D=64, F=96))
    with pytest.raises(GraphError, match="broadcast Add"):
        ex.DeviceExecutor(m2, cuda_device)


def test_graph_replay_matches_eager(cuda_device):
    """use_graph: the first run records the node launches, later runs replay them."""
    m = ex.fuse_matmulq_epilogues(ex.quantize_matmuls(mlp_model(M=8, D=768, F=3072)))
    eager = ex.DeviceExecutor(m, cuda_device, mode="fp32")
    graphed = ex.DeviceExecutor(m, cuda_device, mode="fp32", use_graph=True)
    rng = np.random.default_rng(3)
    for i in range(3):
        x = rng.standard_normal((8, 768)).astype(np.float32)
        want = eager.run(x)[0]
        got = graphed.run(x)[0]
        assert np.array_equal(got, want), f"run {i}"
    assert graphed.graph is not None


def test_reference_fused_graph_runs(cuda_device):
    """FusedMatMulBiasGeluTanh from the reference's fusion pass runs as one MatMulQ."""
    m = mlp_model(M=4, D=768, F=3072, seed=9)
    g = m.graph
    mm, add, gelu = g.nodes[1], g.nodes[2], g.nodes[3]
    ref_model = ex.LoadedModel(ex.Graph(list(g.tensors), list(g.nodes), list(g.inputs), list(g.outputs)),
                               dict(m.weights))
    g.nodes[1:4] = [Node("FusedMatMulBiasGeluTanh", [mm.inputs[0], mm.inputs[1], add.inputs[1]],
                         list(gelu.outputs))]
    run_model = ex.fuse_matmulq_epilogues(ex.quantize_matmuls(m))
    x = np.random.default_rng(9).standard_normal((4, 768)).astype(np.float32)
    y = ex.DeviceExecutor(run_model, cuda_device, mode="fp32").run(x)[0]
    assert rel_err(y, reference_forward(ref_model, x)) <= 1e-4


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_block_chain_with_arena_residual(cuda_device, mode):
    """Three chained blocks: from the second on, the residual a fused MatMulQ adds is
    an intermediate in the arena, so its bytes must survive until that MatMulQ."""
    m = block_chain(n_blocks=3, M=8, D=768, F=3072, seed=5)
    run_model = ex.fuse_matmulq_epilogues(ex.quantize_matmuls(m))
    assert sum(n.attrs.get("epilogue") == "residual" for n in run_model.graph.nodes) == 3
    x = np.random.default_rng(5).standard_normal((8, 768)).astype(np.float32)
    y = ex.DeviceExecutor(run_model, cuda_device, mode=mode).run(x)[0]
    err = rel_err(y, reference_forward(m, x))
    assert err <= (1e-4 if mode == "fp32" else 2e-2), f"rel err {err:.3e}"
