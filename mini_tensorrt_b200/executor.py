"""Host mirror of the reference's model plumbing for MatMulQ on the device.

The reference runs a model as: load a JSON graph and its weights blob
(src/frontend/json/json_loader.cpp:53-133), optionally rewrite it
(src/optimizer/fusion.cpp:22-130), plan one arena for the intermediate tensors
(src/memory/memory_planner.cpp:19-85) and execute the nodes in topological order
(src/graph/graph.cpp:32-91), on the CPU or with the CUDA executor
(backends/cuda/cuda_executor.cpp:36-160). For MatMulQ that chain breaks in three
places: the loader copies every weight through `data<float>()` (:104), which aborts
on int8 weights in Debug builds; the CUDA executor uploads weights the same way
(:67-69) and throws on MatMulQ (:152-154); and nothing turns an fp32 MatMul into a
MatMulQ. This module keeps the reference's names, file format and error behaviour
(GraphError at set-up) and closes those gaps:

* `load_json_model` reads the same JSON + blob format, copying each weight's bytes
  as its own dtype (f32, i32 or i8);
* `quantize_matmuls` rewrites MatMul(x, W) with an fp32 weight W [K, N] into
  MatMulQ(x, Wq, scale) with the reference packer (per output channel,
  scale = max|W[:, j]| / 127, q = lround(W / scale));
* `fuse_matmulq_epilogues` folds MatMulQ -> Add(bias) [-> GeluTanh] and MatMulQ ->
  Add(same-shape residual) into one MatMulQ node whose epilogue does the rest
  (the int8 analogue of fuse_matmul_bias_gelu);
* `plan_memory` is the reference's greedy-by-size lifetime planner with byte sizes
  per dtype and a 256-byte alignment (the reference arena is fp32-only and
  16-byte aligned);
* `DeviceExecutor` uploads and pre-packs the weights, places every intermediate in
  one device arena, sizes one MatMulQ workspace, all at construction, so that
  `run()` allocates no device memory; it dispatches MatMulQ to libmtrtq and the
  element-wise ops (Add, LayerNorm, GeluTanh) to the library's device kernels.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from ._lib import check, lib
from .matmulq import MODES, PackedWeight, Workspace, quantize_per_channel, workspace_bytes
from .registry import GraphError, Node

KINDS = ("input", "output", "weight", "intermediate")
DTYPES = {"f32": np.float32, "i32": np.int32, "i8": np.int8}
TORCH_DTYPES = {"f32": torch.float32, "i32": torch.int32, "i8": torch.int8}
ARENA_ALIGNMENT = 256  # bytes: TMA and 16-byte vector loads need at least 16


@dataclass
class TensorInfo:
    """include/mtrt/graph.h: name, dtype ("f32" | "i32" | "i8"), shape, kind."""
    name: str
    dtype: str
    shape: tuple
    kind: str

    @property
    def nbytes(self) -> int:
        return int(np.prod(self.shape, dtype=np.int64)) * np.dtype(DTYPES[self.dtype]).itemsize


# Attributes of a fused MatMulQ that name tensors it reads in its epilogue.
EPILOGUE_OPERANDS = ("bias", "residual")


def node_reads(nd) -> list:
    """Every tensor a node reads: its inputs, then the epilogue operands a fused
    MatMulQ names in its attributes (bias, residual). Ordering, consumer counts
    and arena lifetimes all go through this, so a tensor read only by an
    epilogue is ordered before its reader and stays live until it has run."""
    reads = list(nd.inputs)
    for k in EPILOGUE_OPERANDS:
        if k in nd.attrs:
            reads.append(int(nd.attrs[k]))
    return reads


@dataclass
class Graph:
    tensors: list = field(default_factory=list)   # TensorInfo, indexed by tensor id
    nodes: list = field(default_factory=list)     # registry.Node, inputs/outputs are tensor ids
    inputs: list = field(default_factory=list)
    outputs: list = field(default_factory=list)

    def add_tensor(self, info: TensorInfo) -> int:
        self.tensors.append(info)
        return len(self.tensors) - 1

    def topo_order(self) -> list:
        """Kahn's algorithm in node order, as src/graph/graph.cpp:32-91: one
        producer per tensor, tensors read but never written must be inputs or
        weights, no cycles."""
        n = len(self.nodes)
        producer = [-1] * len(self.tensors)
        for ni, nd in enumerate(self.nodes):
            for t in nd.outputs:
                if not 0 <= t < len(self.tensors):
                    raise GraphError("node writes out-of-range tensor id")
                if producer[t] != -1:
                    raise GraphError("tensor has more than one producer (not SSA-like)")
                producer[t] = ni
        indeg = [0] * n
        consumers = [[] for _ in range(n)]
        for ni, nd in enumerate(self.nodes):
            for t in node_reads(nd):
                if not 0 <= t < len(self.tensors):
                    raise GraphError("node reads out-of-range tensor id")
                p = producer[t]
                if p == -1:
                    if self.tensors[t].kind not in ("input", "weight"):
                        raise GraphError(f"tensor consumed but never produced: {self.tensors[t].name}")
                else:
                    consumers[p].append(ni)
                    indeg[ni] += 1
        ready = [ni for ni in range(n) if indeg[ni] == 0]
        order = []
        while ready:
            ni = ready.pop(0)
            order.append(ni)
            for d in consumers[ni]:
                indeg[d] -= 1
                if indeg[d] == 0:
                    ready.append(d)
        if len(order) != n:
            raise GraphError("graph contains a cycle")
        return order


@dataclass
class LoadedModel:
    graph: Graph
    weights: dict  # tensor id -> numpy array (dtype and shape of its TensorInfo)


def load_json_model(path: str) -> LoadedModel:
    """The reference's JSON model (src/frontend/json/json_loader.cpp:53-133): tensors
    {name, dtype, shape, kind[, offset, nbytes]}, nodes {op, inputs, outputs[,
    attrs]}, graph inputs and outputs, weights in the blob named by
    "weights_file". Each weight is read as its own dtype (the reference reads every
    weight through data<float>(), :104). Errors raise GraphError as the reference's
    loader does."""
    try:
        with open(path) as f:
            j = json.load(f)
    except OSError:
        raise GraphError(f"cannot open JSON model: {path}")
    except ValueError as e:
        raise GraphError(f"JSON parse error: {e}")
    blob = b""
    if "weights_file" in j:
        bin_path = os.path.join(os.path.dirname(path) or ".", j["weights_file"])
        try:
            with open(bin_path, "rb") as f:
                blob = f.read()
        except OSError:
            raise GraphError(f"cannot open weights file: {bin_path}")
    g = Graph()
    ids = {}
    weights = {}
    for jt in j["tensors"]:
        if jt["dtype"] not in DTYPES:
            raise GraphError(f"unsupported dtype in JSON model: {jt['dtype']}")
        if jt["kind"] not in KINDS:
            raise GraphError(f"unknown tensor kind in JSON model: {jt['kind']}")
        info = TensorInfo(jt["name"], jt["dtype"], tuple(int(d) for d in jt["shape"]), jt["kind"])
        if info.name in ids:
            raise GraphError(f"duplicate tensor name in JSON model: {info.name}")
        tid = g.add_tensor(info)
        ids[info.name] = tid
        if info.kind == "weight":
            off, nb = int(jt["offset"]), int(jt["nbytes"])
            if off + nb > len(blob):
                raise GraphError(f"weight '{info.name}' exceeds weights blob")
            if nb != info.nbytes:
                raise GraphError(f"weight '{info.name}' byte size mismatch")
            weights[tid] = np.frombuffer(blob, dtype=DTYPES[info.dtype], count=nb // np.dtype(
                DTYPES[info.dtype]).itemsize, offset=off).reshape(info.shape).copy()

    def id_of(name):
        if name not in ids:
            raise GraphError(f"node references unknown tensor: {name}")
        return ids[name]

    for jn in j["nodes"]:
        attrs = {}
        for k, v in (jn.get("attrs") or {}).items():
            if isinstance(v, bool) or not isinstance(v, (int, float, list)):
                raise GraphError("unsupported attribute type in JSON model")
            attrs[k] = [int(e) for e in v] if isinstance(v, list) else v
        g.nodes.append(Node(jn["op"], [id_of(t) for t in jn["inputs"]], [id_of(t) for t in jn["outputs"]],
                            attrs))
    g.inputs = [id_of(t) for t in j["inputs"]]
    g.outputs = [id_of(t) for t in j["outputs"]]
    return LoadedModel(g, weights)


def save_json_model(model: LoadedModel, path: str, weights_file: str | None = None) -> None:
    """Writes a model in the same format (weights concatenated into one blob)."""
    g = model.graph
    weights_file = weights_file or os.path.splitext(os.path.basename(path))[0] + ".bin"
    blob = bytearray()
    tensors = []
    for tid, t in enumerate(g.tensors):
        jt = {"name": t.name, "dtype": t.dtype, "shape": list(t.shape), "kind": t.kind}
        if t.kind == "weight":
            data = np.ascontiguousarray(model.weights[tid], dtype=DTYPES[t.dtype]).tobytes()
            jt["offset"], jt["nbytes"] = len(blob), len(data)
            blob += data
        tensors.append(jt)
    nodes = [{"op": n.op_type, "inputs": [g.tensors[t].name for t in n.inputs],
              "outputs": [g.tensors[t].name for t in n.outputs], **({"attrs": n.attrs} if n.attrs else {})}
             for n in g.nodes]
    with open(os.path.join(os.path.dirname(path) or ".", weights_file), "wb") as f:
        f.write(bytes(blob))
    with open(path, "w") as f:
        json.dump({"weights_file": weights_file, "tensors": tensors, "nodes": nodes,
                   "inputs": [g.tensors[t].name for t in g.inputs],
                   "outputs": [g.tensors[t].name for t in g.outputs]}, f)


def _consumers(g: Graph) -> dict:
    out = {}
    for ni, nd in enumerate(g.nodes):
        for t in node_reads(nd):
            out.setdefault(t, []).append(ni)
    return out


def quantize_matmuls(model: LoadedModel) -> LoadedModel:
    """MatMul(x, W) with W an fp32 weight [K, N] -> MatMulQ(x, Wq, scale): Wq int8
    [K, N] and scale f32 [N] by the reference packer (tests/golden_kernel_test.cpp:
    163-170; an all-zero column is rejected). A FusedMatMulBiasGeluTanh(x, W, bias)
    left by the reference's own fusion pass (src/optimizer/fusion.cpp:91-93) becomes
    MatMulQ {bias, epilogue "gelu"}. Other nodes are kept; the fp32 weight is dropped
    when nothing else reads it."""
    g = model.graph
    out = Graph(list(g.tensors), [], list(g.inputs), list(g.outputs))
    weights = dict(model.weights)
    cons = _consumers(g)
    for nd in g.nodes:
        fused_gelu = nd.op_type == "FusedMatMulBiasGeluTanh" and len(nd.inputs) == 3
        if (nd.op_type == "MatMul" and len(nd.inputs) == 2) or fused_gelu:
            w_id = nd.inputs[1]
            info = g.tensors[w_id]
            if info.kind == "weight" and info.dtype == "f32" and len(info.shape) == 2:
                q, s = quantize_per_channel(model.weights[w_id])
                qi = out.add_tensor(TensorInfo(info.name + ".q8", "i8", info.shape, "weight"))
                si = out.add_tensor(TensorInfo(info.name + ".scale", "f32", (info.shape[1],), "weight"))
                weights[qi], weights[si] = q, s
                attrs = dict(nd.attrs)
                if fused_gelu:
                    attrs.update(bias=nd.inputs[2], epilogue="gelu")
                out.nodes.append(Node("MatMulQ", [nd.inputs[0], qi, si], list(nd.outputs), attrs))
                if len(cons.get(w_id, [])) == 1:
                    weights.pop(w_id, None)
                continue
        out.nodes.append(Node(nd.op_type, list(nd.inputs), list(nd.outputs), dict(nd.attrs)))
    return LoadedModel(out, weights)


def fuse_matmulq_epilogues(model: LoadedModel) -> LoadedModel:
    """Folds, as src/optimizer/fusion.cpp:22-130 does for fp32 MatMul + Add + Gelu,
    a MatMulQ whose output is a single-use intermediate into the Add that reads it
    and, after a bias Add, into a GeluTanh that reads the sum:
      MatMulQ -> Add(bias [N])             => MatMulQ {bias}
      MatMulQ -> Add(bias [N]) -> GeluTanh => MatMulQ {bias, epilogue "gelu"}
      MatMulQ -> Add(r, same shape)        => MatMulQ {epilogue "residual", residual r}
    The folded node writes the last node's output. Intermediates that no longer
    have a producer are left unused (not planned)."""
    g = model.graph
    cons = _consumers(g)
    outs = set(g.outputs)
    nodes = g.nodes

    def single_use(t):
        return g.tensors[t].kind == "intermediate" and len(cons.get(t, [])) == 1 and t not in outs

    fused, drop = {}, set()
    for ni, mm in enumerate(nodes):
        if mm.op_type != "MatMulQ" or len(mm.outputs) != 1 or "bias" in mm.attrs:
            continue
        t0 = mm.outputs[0]
        if not single_use(t0):
            continue
        ai = cons[t0][0]
        add = nodes[ai]
        if add.op_type != "Add" or len(add.inputs) != 2 or t0 not in add.inputs or \
                add.inputs[0] == add.inputs[1]:
            continue
        first = add.inputs[0] == t0
        other = add.inputs[1] if first else add.inputs[0]
        t1 = add.outputs[0]
        o_info, t_info = g.tensors[other], g.tensors[t0]
        n_out = t_info.shape[-1]
        attrs = dict(mm.attrs)
        # a bias broadcasts only as the Add's second input (kernels_elementwise.cpp:20, :31-35)
        if first and o_info.kind == "weight" and o_info.dtype == "f32" and int(np.prod(o_info.shape)) == n_out \
                and tuple(o_info.shape) != tuple(t_info.shape):
            attrs["bias"] = other
            end, dropped = t1, [ai]
            if single_use(t1) and nodes[cons[t1][0]].op_type == "GeluTanh":
                gi = cons[t1][0]
                attrs["epilogue"] = "gelu"
                end, dropped = nodes[gi].outputs[0], [ai, gi]
        elif tuple(o_info.shape) == tuple(t_info.shape) and o_info.dtype == "f32":
            attrs["epilogue"] = "residual"
            attrs["residual"] = other
            end, dropped = t1, [ai]
        else:
            continue
        fused[ni] = Node("MatMulQ", list(mm.inputs), [end], attrs)
        drop.update(dropped)
    out = Graph(list(g.tensors), [], list(g.inputs), list(g.outputs))
    for ni, nd in enumerate(nodes):
        if ni in drop:
            continue
        out.nodes.append(fused.get(ni, Node(nd.op_type, list(nd.inputs), list(nd.outputs), dict(nd.attrs))))
    return LoadedModel(out, dict(model.weights))


@dataclass
class MemoryPlan:
    offset: dict        # tensor id -> byte offset in the arena
    total_bytes: int
    intervals: list     # (tensor id, first_write, last_read, nbytes)


def plan_memory(g: Graph, alignment: int = ARENA_ALIGNMENT) -> MemoryPlan:
    """src/memory/memory_planner.cpp:19-85 over every dtype: live interval of each
    produced intermediate over the topological order (written at its producer's
    step, live through its last reader's), then greedy by size (ties by id): each
    tensor takes the lowest aligned offset that fits between the byte ranges of
    already placed tensors whose intervals overlap its own."""
    order = g.topo_order()
    live = {}
    for step, ni in enumerate(order):
        nd = g.nodes[ni]
        for t in nd.outputs:
            if g.tensors[t].kind == "intermediate" and t not in live:
                live[t] = [step, step]
        for t in node_reads(nd):
            if t in live:
                live[t][1] = step
    ivs = sorted(((t, a, b, g.tensors[t].nbytes) for t, (a, b) in live.items()), key=lambda x: (-x[3], x[0]))
    up = lambda x: (x + alignment - 1) // alignment * alignment
    placed, offset, total = [], {}, 0
    for t, a, b, nb in ivs:
        blocked = sorted((o, o + n) for (o, n, pa, pb) in placed if a <= pb and pa <= b)
        off = 0
        for bb, be in blocked:
            if off + nb <= bb:
                break
            off = max(off, up(be))
        offset[t] = off
        placed.append((off, nb, a, b))
        total = max(total, off + nb)
    return MemoryPlan(offset, up(total), ivs)


class DeviceExecutor:
    """Runs a LoadedModel on one GPU, as the reference's CudaExecutor does
    (backends/cuda/cuda_executor.cpp:36-160), with MatMulQ on libmtrtq.

    Construction (set-up, may allocate): checks every node is supported (GraphError
    otherwise), uploads the weights (MatMulQ weights pre-packed once), places the
    intermediates in one arena by `plan_memory`, gives inputs and outputs their own
    buffers with pinned host staging, and sizes one zero-filled MatMulQ workspace.
    `run(*inputs)` copies the inputs in, launches the nodes in topological order on
    the executor's stream and returns the outputs as numpy arrays; it allocates no
    device memory.

    mode: MatMulQ mode ("bf16" rounds activations to bf16; "fp32" keeps them).
    use_graph: record the node launches of the first run() as a CUDA graph and
    replay it in later runs (the inputs, arena and outputs keep their addresses, so
    one recording serves every run); the copies in and out stay outside the graph.
    """

    SUPPORTED = ("MatMulQ", "Add", "LayerNorm", "GeluTanh")

    def __init__(self, model: LoadedModel, device="cuda", mode: str = "bf16", use_graph: bool = False):
        self.model, self.g, self.mode = model, model.graph, mode
        self.use_graph, self.graph = use_graph, None
        self.dev = torch.device(device)
        self.order = self.g.topo_order()
        self.stream = torch.cuda.Stream(self.dev)
        g = self.g
        for ni in self.order:
            nd = g.nodes[ni]
            if nd.op_type not in self.SUPPORTED:
                raise GraphError(f"DeviceExecutor: unsupported op '{nd.op_type}'")
            self._check_node(nd)
        self.plan = plan_memory(g)
        self.arena = torch.zeros(max(self.plan.total_bytes, 1), dtype=torch.uint8, device=self.dev)
        self.buf = {}
        self.host = {}
        # Weights the nodes read directly (a MatMulQ's int8 weight is uploaded packed, below).
        read = set()
        for ni in self.order:
            nd = g.nodes[ni]
            read.update(nd.inputs[2:] if nd.op_type == "MatMulQ" else nd.inputs)
            if nd.op_type == "MatMulQ":
                read.add(nd.inputs[0])
                read.update(nd.attrs[k] for k in ("bias", "residual") if k in nd.attrs)
        for tid, t in enumerate(g.tensors):
            if t.kind == "intermediate" and tid in self.plan.offset:
                off = self.plan.offset[tid]
                self.buf[tid] = self.arena[off:off + t.nbytes].view(TORCH_DTYPES[t.dtype]).view(t.shape)
            elif t.kind == "weight" and tid in read:
                if tid not in model.weights:
                    raise GraphError(f"weight '{t.name}' has no data")
                self.buf[tid] = torch.from_numpy(np.ascontiguousarray(model.weights[tid])).to(self.dev)
            elif t.kind in ("input", "output"):
                self.buf[tid] = torch.zeros(t.shape, dtype=TORCH_DTYPES[t.dtype], device=self.dev)
                self.host[tid] = torch.zeros(t.shape, dtype=TORCH_DTYPES[t.dtype]).pin_memory()
        # MatMulQ weights: packed once (the weight upload of the reference's ctor, :61-72).
        self.packed = {}
        need = 0
        for ni in self.order:
            nd = g.nodes[ni]
            if nd.op_type == "MatMulQ":
                x, wq, sc = nd.inputs
                key = (wq, sc)
                if key not in self.packed:
                    self.packed[key] = PackedWeight.from_int8(torch.from_numpy(model.weights[wq]),
                                                              torch.from_numpy(model.weights[sc]), self.dev)
                K, N = g.tensors[wq].shape
                M = int(np.prod(g.tensors[x].shape)) // K
                need = max(need, workspace_bytes(M, K, N, torch.float32, mode))
        self.ws = Workspace(self.dev).get(need)
        torch.cuda.synchronize(self.dev)

    def _check_node(self, nd):
        g = self.g
        T = lambda i: g.tensors[i]
        if nd.op_type == "MatMulQ":
            if len(nd.inputs) != 3 or len(nd.outputs) != 1:
                raise GraphError("MatMulQ expects A, W_int8, scale and one output")
            x, wq, sc = (T(i) for i in nd.inputs)
            if wq.kind != "weight" or wq.dtype != "i8" or len(wq.shape) != 2:
                raise GraphError("MatMulQ: W must be an i8 weight [K, N] on the device")
            if sc.kind != "weight" or sc.dtype != "f32" or int(np.prod(sc.shape)) != wq.shape[1]:
                raise GraphError("MatMulQ scale must be per-column [N]")
            if x.dtype != "f32" or x.shape[-1] != wq.shape[0]:
                raise GraphError("MatMulQ inner dimensions disagree")
            y = T(nd.outputs[0])
            M = int(np.prod(x.shape)) // wq.shape[0]
            if int(np.prod(y.shape)) != M * wq.shape[1] or y.shape[-1] != wq.shape[1]:
                raise GraphError("MatMulQ output shape wrong")
            if "bias" in nd.attrs:
                b = T(nd.attrs["bias"])
                if b.dtype != "f32" or int(np.prod(b.shape)) != wq.shape[1]:
                    raise GraphError("MatMulQ bias must be f32 [N]")
            if nd.attrs.get("epilogue") == "residual":
                r = T(nd.attrs["residual"])
                if tuple(r.shape) != tuple(y.shape) or r.dtype != "f32":
                    raise GraphError("MatMulQ residual must match the output")
        elif nd.op_type == "Add":
            a, b = (T(i) for i in nd.inputs)
            if tuple(a.shape) != tuple(b.shape):
                # the reference's broadcast form (kernels_elementwise.cpp:31-35) runs on the
                # device only folded into a MatMulQ (fuse_matmulq_epilogues)
                raise GraphError("DeviceExecutor: a broadcast Add must follow a MatMulQ")
        elif nd.op_type == "LayerNorm":
            if len(nd.inputs) != 3 or "eps" not in nd.attrs:
                raise GraphError("LayerNorm expects x, gamma, beta and an eps attribute")
            x, gm, bt = (T(i) for i in nd.inputs)
            if int(np.prod(gm.shape)) != x.shape[-1] or int(np.prod(bt.shape)) != x.shape[-1]:
                raise GraphError("LayerNorm gamma/beta size")

    def _launch(self, nd):
        g, sp, L = self.g, self.stream.cuda_stream, lib()
        B = self.buf
        if nd.op_type == "MatMulQ":
            x, wq, sc = nd.inputs
            K, N = g.tensors[wq].shape
            M = B[x].numel() // K
            pw = self.packed[(wq, sc)]
            y = B[nd.outputs[0]]
            bias = B[nd.attrs["bias"]] if "bias" in nd.attrs else None
            epi = {"gelu": _lib.EPILOGUE_GELU_TANH, "residual": _lib.EPILOGUE_ADD_RESIDUAL}.get(
                nd.attrs.get("epilogue"), _lib.EPILOGUE_NONE)
            res = B[nd.attrs["residual"]] if epi == _lib.EPILOGUE_ADD_RESIDUAL else None
            ws = self.ws
            check(L.mtrtq_matmul_ex(B[x].data_ptr(), _lib.DTYPE_F32, K, pw.packed.data_ptr(), pw.scale.data_ptr(),
                                    bias.data_ptr() if bias is not None else None, y.data_ptr(), N, M, K, N,
                                    MODES[self.mode], ws.data_ptr() if ws is not None else None,
                                    ws.numel() if ws is not None else 0, epi,
                                    res.data_ptr() if res is not None else None, N if res is not None else 0, sp),
                  "MatMulQ")
        elif nd.op_type == "Add":
            a, b = (B[i] for i in nd.inputs)
            y = B[nd.outputs[0]]
            if y.data_ptr() != a.data_ptr():
                y.copy_(a)
            check(L.mtrtq_add_inplace(y.data_ptr(), b.data_ptr(), y.numel(), sp), "Add")
        elif nd.op_type == "LayerNorm":
            x, gm, bt = (B[i] for i in nd.inputs)
            D = x.shape[-1]
            check(L.mtrtq_layernorm(x.data_ptr(), gm.data_ptr(), bt.data_ptr(), B[nd.outputs[0]].data_ptr(),
                                    x.numel() // D, D, float(nd.attrs["eps"]), sp), "LayerNorm")
        elif nd.op_type == "GeluTanh":
            x = B[nd.inputs[0]]
            check(L.mtrtq_gelu_tanh(x.data_ptr(), B[nd.outputs[0]].data_ptr(), x.numel(), sp), "GeluTanh")

    def run(self, *inputs):
        """inputs: one array per graph input (its shape and dtype). Returns a list of
        numpy arrays, one per graph output."""
        g = self.g
        if len(inputs) != len(g.inputs):
            raise GraphError(f"run expects {len(g.inputs)} inputs")
        with torch.cuda.stream(self.stream):
            for tid, arr in zip(g.inputs, inputs):
                h = self.host[tid]
                h.numpy()[...] = np.asarray(arr).reshape(h.shape)
                self.buf[tid].copy_(h, non_blocking=True)
            if self.graph is not None:
                self.graph.replay()
            else:
                for ni in self.order:
                    self._launch(g.nodes[ni])
            for tid in g.outputs:
                self.host[tid].copy_(self.buf[tid], non_blocking=True)
        self.stream.synchronize()
        out = [self.host[tid].numpy().copy() for tid in g.outputs]
        if self.use_graph and self.graph is None:
            # record after one eager run (first launches do per-device set-up)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=self.stream):
                for ni in self.order:
                    self._launch(g.nodes[ni])
            self.stream.synchronize()
            self.graph = graph
        return out
