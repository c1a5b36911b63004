"""EP-core bindings (include/b200ep_ep.h): describe a graph, let the EP claim and partition it,
compile the partitions into device plans and run them.

``GraphBuilder`` plays the part of the reference tests' ONNX-IR builders (tests/ops/_models.py):
typed values, initializers, nodes with attributes.  ``Session`` plays ONNX Runtime's part for
graphs the EP claims completely: it runs the compiled partitions in order and hands boundary
tensors between them on the device.
"""

from __future__ import annotations

import ctypes
from typing import Any

import numpy as np

from . import B200EPError, check, load_library

DT = {np.dtype(np.float32): 1, np.dtype(np.uint8): 2, np.dtype(np.int8): 3, np.dtype(np.int32): 6,
      np.dtype(np.int64): 7, np.dtype(np.float16): 10}
FLOAT, UINT8, INT32, INT64, FLOAT16, BFLOAT16 = 1, 2, 6, 7, 10, 16
MAX_RANK = 8


class Tensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("dims", ctypes.c_int64 * MAX_RANK), ("on_device", ctypes.c_int32)]


_configured = False


def _lib():
    global _configured
    L = load_library()
    if not _configured:
        vp, cp, i32, i64, sz = ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
        P64 = ctypes.POINTER(ctypes.c_int64)
        L.b200ep_graph_create.restype = vp
        L.b200ep_graph_release.argtypes = [vp]
        L.b200ep_graph_set_opset.argtypes = [vp, cp, i32]
        for f in (L.b200ep_graph_add_value, L.b200ep_graph_add_input, L.b200ep_graph_add_output):
            f.argtypes = [vp, cp, i32, i32, P64]
        L.b200ep_graph_add_initializer.argtypes = [vp, cp, i32, i32, P64, vp, sz]
        L.b200ep_graph_add_node.argtypes = [vp, cp, cp, cp, i32, ctypes.POINTER(cp), i32, ctypes.POINTER(cp),
                                            ctypes.POINTER(ctypes.c_int)]
        L.b200ep_graph_node_attr_int.argtypes = [vp, i32, cp, i64]
        L.b200ep_graph_node_attr_float.argtypes = [vp, i32, cp, ctypes.c_float]
        L.b200ep_graph_node_attr_string.argtypes = [vp, i32, cp, cp]
        L.b200ep_graph_node_attr_ints.argtypes = [vp, i32, cp, P64, i32]
        L.b200ep_graph_set_metadata.argtypes = [vp, cp, cp]
        L.b200ep_graph_num_nodes.argtypes = [vp]
        L.b200ep_ep_create.restype = vp
        L.b200ep_ep_create.argtypes = [ctypes.POINTER(cp), ctypes.POINTER(cp), sz]
        L.b200ep_ep_release.argtypes = [vp]
        L.b200ep_ep_name.argtypes = [vp]
        L.b200ep_ep_name.restype = cp
        L.b200ep_ep_get_capability.argtypes = [vp, vp, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32)]
        L.b200ep_ep_claim_reason.argtypes = [vp, i32]
        L.b200ep_ep_claim_reason.restype = cp
        L.b200ep_ep_compile.argtypes = [vp, vp, i32, ctypes.POINTER(vp)]
        L.b200ep_compiled_release.argtypes = [vp]
        L.b200ep_compiled_num_inputs.argtypes = [vp]
        L.b200ep_compiled_num_outputs.argtypes = [vp]
        L.b200ep_compiled_input_name.argtypes = [vp, i32]
        L.b200ep_compiled_input_name.restype = cp
        L.b200ep_compiled_output_name.argtypes = [vp, i32]
        L.b200ep_compiled_output_name.restype = cp
        L.b200ep_compiled_output_shapes.argtypes = [vp, ctypes.POINTER(Tensor), sz, ctypes.POINTER(Tensor), sz]
        L.b200ep_compiled_run.argtypes = [vp, ctypes.POINTER(Tensor), sz, ctypes.POINTER(Tensor), sz, vp]
        L.b200ep_compiled_describe.argtypes = [vp]
        L.b200ep_compiled_describe.restype = cp
        L.b200ep_compiled_launches_per_run.argtypes = [vp]
        L.b200ep_tp_unique_id.argtypes = [vp]
        L.b200ep_ep_set_tensor_parallel.argtypes = [vp, i32, i32, vp]
        L.b200ep_tp_shard_preview.argtypes = [vp, i32, i32, ctypes.c_char_p, sz, ctypes.POINTER(sz)]
        L.b200ep_ep_summary.argtypes = [vp, ctypes.c_char_p, sz, ctypes.POINTER(sz)]
        _configured = True
    return L


def _dims(shape):
    arr = (ctypes.c_int64 * max(1, len(shape)))(*[int(d) for d in shape])
    return arr


def _cstrs(names):
    arr = (ctypes.c_char_p * max(1, len(names)))(*[n.encode() for n in names])
    return arr


class GraphBuilder:
    """Builds a graph through the C ABI.  Values: ``tensor`` (typed value), ``input``, ``output``,
    ``initializer``; ``node`` appends a node (topological order) and returns its index."""

    def __init__(self, opset: int = 24, ms_opset: int = 1):
        L = _lib()
        self._g = L.b200ep_graph_create()
        if not self._g:
            raise MemoryError("b200ep_graph_create failed")
        self.opset(None, opset)
        self.opset("com.microsoft", ms_opset)
        self.node_names: list[str] = []
        self.inputs: list[tuple[str, int, tuple]] = []
        self.outputs: list[tuple[str, int, tuple]] = []

    def __del__(self):
        g = getattr(self, "_g", None)
        if g:
            _lib().b200ep_graph_release(g)
            self._g = None

    @property
    def handle(self):
        return self._g

    def opset(self, domain, version):
        check(_lib().b200ep_graph_set_opset(self._g, (domain or "").encode(), version))

    def tensor(self, name, dtype, shape):
        check(_lib().b200ep_graph_add_value(self._g, name.encode(), dtype, len(shape), _dims(shape)))
        return name

    def input(self, name, dtype, shape):
        check(_lib().b200ep_graph_add_input(self._g, name.encode(), dtype, len(shape), _dims(shape)))
        self.inputs.append((name, dtype, tuple(shape)))
        return name

    def output(self, name, dtype, shape):
        check(_lib().b200ep_graph_add_output(self._g, name.encode(), dtype, len(shape), _dims(shape)))
        self.outputs.append((name, dtype, tuple(shape)))
        return name

    def initializer(self, name, array: np.ndarray, dtype: int | None = None):
        a = np.ascontiguousarray(array)
        code = dtype if dtype is not None else DT[a.dtype]
        check(_lib().b200ep_graph_add_initializer(self._g, name.encode(), code, a.ndim, _dims(a.shape),
                                                  a.ctypes.data_as(ctypes.c_void_p), a.nbytes))
        return name

    def node(self, op_type, inputs, outputs, *, domain="", name="", **attrs) -> int:
        idx = ctypes.c_int(-1)
        check(_lib().b200ep_graph_add_node(self._g, op_type.encode(), domain.encode(), name.encode(), len(inputs),
                                           _cstrs(inputs), len(outputs), _cstrs(outputs), ctypes.byref(idx)))
        for k, v in attrs.items():
            if isinstance(v, bool) or isinstance(v, (int, np.integer)):
                check(_lib().b200ep_graph_node_attr_int(self._g, idx.value, k.encode(), int(v)))
            elif isinstance(v, (float, np.floating)):
                check(_lib().b200ep_graph_node_attr_float(self._g, idx.value, k.encode(), float(v)))
            elif isinstance(v, str):
                check(_lib().b200ep_graph_node_attr_string(self._g, idx.value, k.encode(), v.encode()))
            else:
                vals = [int(x) for x in v]
                arr = (ctypes.c_int64 * max(1, len(vals)))(*vals)
                check(_lib().b200ep_graph_node_attr_ints(self._g, idx.value, k.encode(), arr, len(vals)))
        self.node_names.append(name or op_type)
        return idx.value

    def metadata(self, key, value):
        check(_lib().b200ep_graph_set_metadata(self._g, key.encode(), value.encode()))

    def num_nodes(self) -> int:
        return _lib().b200ep_graph_num_nodes(self._g)


class ExecutionProvider:
    def __init__(self, **options: Any):
        L = _lib()
        keys = [k for k in options]
        vals = [str(int(v)) if isinstance(v, bool) else str(v) for v in options.values()]
        self._ep = L.b200ep_ep_create(_cstrs(keys), _cstrs(vals), len(keys))
        if not self._ep:
            raise MemoryError("b200ep_ep_create failed")

    def __del__(self):
        ep = getattr(self, "_ep", None)
        if ep:
            _lib().b200ep_ep_release(ep)
            self._ep = None

    @property
    def name(self) -> str:
        return _lib().b200ep_ep_name(self._ep).decode()

    def get_capability(self, g: GraphBuilder):
        n = g.num_nodes()
        groups = (ctypes.c_int32 * max(1, n))()
        num = ctypes.c_int32(0)
        check(_lib().b200ep_ep_get_capability(self._ep, g.handle, groups, ctypes.byref(num)))
        return [int(groups[i]) for i in range(n)], num.value

    def claim_reason(self, node: int) -> str:
        return _lib().b200ep_ep_claim_reason(self._ep, node).decode()

    def summary(self) -> dict:
        """Session summary: claim rate and unclaimed op types with reasons, compiled partitions,
        runs per path (decode / prefill / general) and execution (graph replay / capture / eager),
        shape-key cache, host boundary bytes, host time (printed at release when verbose)."""
        import json

        need = ctypes.c_size_t(0)
        check(_lib().b200ep_ep_summary(self._ep, None, 0, ctypes.byref(need)))
        buf = ctypes.create_string_buffer(need.value)
        check(_lib().b200ep_ep_summary(self._ep, buf, need.value, ctypes.byref(need)))
        return json.loads(buf.value.decode())

    def compile(self, g: GraphBuilder, group: int) -> "Compiled":
        out = ctypes.c_void_p()
        check(_lib().b200ep_ep_compile(self._ep, g.handle, group, ctypes.byref(out)))
        return Compiled(out.value)

    def set_tensor_parallel(self, rank: int, world: int, unique_id: bytes | None):
        buf = ctypes.create_string_buffer(unique_id, 128) if unique_id else None
        check(_lib().b200ep_ep_set_tensor_parallel(self._ep, rank, world, buf))


def tp_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    check(_lib().b200ep_tp_unique_id(buf))
    return buf.raw


def tp_shard_preview(g: GraphBuilder, rank: int, world: int) -> list:
    """Host-only view of rank `rank`'s tensor-parallel plan of the whole graph (no GPU needed)."""
    import json

    need = ctypes.c_size_t(0)
    check(_lib().b200ep_tp_shard_preview(g.handle, rank, world, None, 0, ctypes.byref(need)))
    buf = ctypes.create_string_buffer(need.value)
    check(_lib().b200ep_tp_shard_preview(g.handle, rank, world, buf, need.value, ctypes.byref(need)))
    return json.loads(buf.value.decode())


def _torch_code(t) -> int:
    import torch

    return {torch.float32: 1, torch.uint8: 2, torch.int8: 3, torch.int32: 6, torch.int64: 7, torch.float16: 10,
            torch.bfloat16: 16}[t.dtype]


def make_tensor(t) -> Tensor:
    """Describe a torch tensor (device or host) or a numpy array (host) for the C ABI."""
    x = Tensor()
    if isinstance(t, np.ndarray):
        assert t.flags.c_contiguous
        x.data = t.ctypes.data
        x.dtype = DT[t.dtype]
        x.on_device = 0
    else:
        assert t.is_contiguous()
        x.data = t.data_ptr()
        x.dtype = _torch_code(t)
        x.on_device = int(t.is_cuda)
    x.rank = len(t.shape)
    for i, d in enumerate(t.shape):
        x.dims[i] = int(d)
    return x


class Compiled:
    def __init__(self, handle):
        self._c = handle

    def __del__(self):
        c = getattr(self, "_c", None)
        if c:
            _lib().b200ep_compiled_release(c)
            self._c = None

    @property
    def input_names(self) -> list[str]:
        L = _lib()
        return [L.b200ep_compiled_input_name(self._c, i).decode() for i in range(L.b200ep_compiled_num_inputs(self._c))]

    @property
    def output_names(self) -> list[str]:
        L = _lib()
        return [L.b200ep_compiled_output_name(self._c, i).decode()
                for i in range(L.b200ep_compiled_num_outputs(self._c))]

    def output_shapes(self, inputs) -> list[tuple[int, tuple]]:
        ins = (Tensor * max(1, len(inputs)))(*[make_tensor(t) for t in inputs])
        n_out = len(self.output_names)
        outs = (Tensor * max(1, n_out))()
        check(_lib().b200ep_compiled_output_shapes(self._c, ins, len(inputs), outs, n_out))
        return [(outs[i].dtype, tuple(outs[i].dims[d] for d in range(outs[i].rank))) for i in range(n_out)]

    def run(self, inputs, outputs, stream=None):
        """inputs/outputs: torch tensors (device or pinned host) or numpy arrays, in name order."""
        ins = (Tensor * max(1, len(inputs)))(*[make_tensor(t) for t in inputs])
        outs = (Tensor * max(1, len(outputs)))(*[make_tensor(t) for t in outputs])
        if stream is None:
            import torch

            stream = torch.cuda.current_stream().cuda_stream
        check(_lib().b200ep_compiled_run(self._c, ins, len(inputs), outs, len(outputs), ctypes.c_void_p(stream)))

    def describe(self) -> str:
        return _lib().b200ep_compiled_describe(self._c).decode()

    def launches_per_run(self) -> int:
        return _lib().b200ep_compiled_launches_per_run(self._c)


TORCH_DT = {1: "float32", 2: "uint8", 6: "int32", 7: "int64", 10: "float16", 16: "bfloat16"}


class Session:
    """Runs a graph the EP claims completely: compiled partitions in order, boundary tensors
    exchanged on the device.  ``run`` takes name -> tensor feeds and optional preallocated
    outputs (e.g. present KV buffers aliasing the past inputs) and returns name -> tensor."""

    def __init__(self, g: GraphBuilder, ep: ExecutionProvider | None = None):
        self.g = g
        self.ep = ep or ExecutionProvider()
        groups, num = self.ep.get_capability(g)
        unclaimed = [i for i, gi in enumerate(groups) if gi < 0]
        if unclaimed:
            reasons = "; ".join(f"{g.node_names[i]}: {self.ep.claim_reason(i)}" for i in unclaimed[:5])
            raise B200EPError(5, f"{len(unclaimed)} node(s) not claimed by the B200 EP ({reasons})")
        self.node_groups = groups
        self.parts = [self.ep.compile(g, i) for i in range(num)]

    def run(self, feeds: dict, outputs: dict | None = None, output_device=True) -> dict:
        import torch

        env = dict(feeds)
        outputs = dict(outputs or {})
        for part in self.parts:
            ins = [env[n] for n in part.input_names]
            shapes = part.output_shapes(ins)
            outs = []
            for name, (dt, shape) in zip(part.output_names, shapes):
                if name in outputs:
                    outs.append(outputs[name])
                else:
                    outs.append(torch.empty(shape, dtype=getattr(torch, TORCH_DT[dt]), device="cuda"))
            part.run(ins, outs)
            env.update(zip(part.output_names, outs))
        return {name: env[name] for name, _, _ in self.g.outputs}
