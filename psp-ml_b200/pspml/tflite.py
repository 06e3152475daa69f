"""TFLite models in and out of the int8 inference path.

The reference's compiler front end parses a .tflite file into its IR
(cargo-psp-ml/src/parse/tflite/lowering.rs:19-124) but never reads the
tensors' quantization parameters and knows no DEPTHWISE_CONV_2D or
AVERAGE_POOL_2D (lowering.rs:92-104).  This module is that front end for
the int8 path:

* `load()` reads a model (`TfliteModel`: tensors with their quantization,
  operators with their options, constant buffers);
* `to_network()` lowers an int8 model whose operators form a chain into a
  `netspec.Network`, the form the C-ABI model, the oracle and the benchmark
  take: CONV_2D, DEPTHWISE_CONV_2D, FULLY_CONNECTED, MAX_POOL_2D,
  AVERAGE_POOL_2D and RESHAPE.  Per-channel multipliers come from the
  scales as TFLite computes them (double product of the float32 scales,
  QuantizeMultiplier), activation ranges as TFLite's
  CalculateActivationRangeQuantized, SAME padding as the reference's
  compute_same_padding (lowering.rs:341-364, extra padding bottom/right);
* `write_network()` writes a `netspec.Network` as an int8 .tflite file (the
  synthetic config networks become loadable models);
* `to_f32_plan()` lowers a float32 model (the reference's mnist-bench
  model) to the op list the f32 C-ABI kernels run, like the reference's
  lowering for its own ops (CONV_2D, MAX_POOL_2D 2x2/2, RESHAPE,
  FULLY_CONNECTED; lowering.rs:156-306).

Operators outside these sets raise ValueError, as the reference's lowering
returns an error for them (lowering.rs:92-104).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from . import capi, flatbuf, netspec

# Schema constants (TFLite schema.fbs: BuiltinOperator, BuiltinOptions union
# order, TensorType, Padding, ActivationFunctionType).
OP_AVERAGE_POOL_2D = 1
OP_CONV_2D = 3
OP_DEPTHWISE_CONV_2D = 4
OP_FULLY_CONNECTED = 9
OP_MAX_POOL_2D = 17
OP_RESHAPE = 22
OP_SOFTMAX = 25

OPT_CONV2D = 1
OPT_DEPTHWISE = 2
OPT_POOL2D = 5
OPT_FULLY_CONNECTED = 8
OPT_RESHAPE = 17

T_FLOAT32, T_INT32, T_UINT8, T_INT64, T_INT8 = 0, 2, 3, 4, 9
PAD_SAME, PAD_VALID = 0, 1
ACT_NONE, ACT_RELU, ACT_RELU_N1_TO_1, ACT_RELU6 = 0, 1, 2, 3

_DTYPE = {T_FLOAT32: np.float32, T_INT32: np.int32, T_UINT8: np.uint8, T_INT64: np.int64,
          T_INT8: np.int8}
_OP_NAMES = {OP_AVERAGE_POOL_2D: "AVERAGE_POOL_2D", OP_CONV_2D: "CONV_2D",
             OP_DEPTHWISE_CONV_2D: "DEPTHWISE_CONV_2D", OP_FULLY_CONNECTED: "FULLY_CONNECTED",
             OP_MAX_POOL_2D: "MAX_POOL_2D", OP_RESHAPE: "RESHAPE", OP_SOFTMAX: "SOFTMAX"}


@dataclass
class TensorInfo:
    shape: tuple
    type: int
    buffer: int
    name: str
    scale: list = field(default_factory=list)
    zero_point: list = field(default_factory=list)
    quantized_dimension: int = 0


@dataclass
class OpInfo:
    code: int
    inputs: list
    outputs: list
    options_type: int
    options: dict

    @property
    def name(self) -> str:
        return _OP_NAMES.get(self.code, f"builtin {self.code}")


@dataclass
class TfliteModel:
    data: bytes
    tensors: list
    operators: list
    inputs: list
    outputs: list
    buffers: list  # (offset, length) into data, or None

    def constant(self, t: int) -> np.ndarray | None:
        ti = self.tensors[t]
        loc = self.buffers[ti.buffer] if ti.buffer < len(self.buffers) else None
        if loc is None:
            return None
        off, n = loc
        dt = np.dtype(_DTYPE[ti.type])
        a = np.frombuffer(self.data, dtype=dt, count=n // dt.itemsize, offset=off)
        return a.reshape(ti.shape) if ti.shape else a


# ------------------------------------------------------------------ reading
def _options(op: flatbuf.Table, otype: int) -> dict:
    t = op.table(4)
    if t is None:
        return {}
    if otype == OPT_CONV2D:
        return dict(padding=t.scalar(0, "b"), stride_w=t.scalar(1, "i"), stride_h=t.scalar(2, "i"),
                    activation=t.scalar(3, "b"), dilation_w=t.scalar(4, "i", 1),
                    dilation_h=t.scalar(5, "i", 1))
    if otype == OPT_DEPTHWISE:
        return dict(padding=t.scalar(0, "b"), stride_w=t.scalar(1, "i"), stride_h=t.scalar(2, "i"),
                    depth_multiplier=t.scalar(3, "i"), activation=t.scalar(4, "b"),
                    dilation_w=t.scalar(5, "i", 1), dilation_h=t.scalar(6, "i", 1))
    if otype == OPT_POOL2D:
        return dict(padding=t.scalar(0, "b"), stride_w=t.scalar(1, "i"), stride_h=t.scalar(2, "i"),
                    filter_w=t.scalar(3, "i"), filter_h=t.scalar(4, "i"),
                    activation=t.scalar(5, "b"))
    if otype == OPT_FULLY_CONNECTED:
        return dict(activation=t.scalar(0, "b"), weights_format=t.scalar(1, "b"),
                    keep_num_dims=t.scalar(2, "?", False))
    if otype == OPT_RESHAPE:
        return dict(new_shape=t.vector(0, "i"))
    return {}


def load(src) -> TfliteModel:
    """Reads a .tflite model from a path or bytes (one subgraph)."""
    data = Path(src).read_bytes() if isinstance(src, (str, Path)) else bytes(src)
    if len(data) < 8:
        raise ValueError("not a TFLite model: too short")
    m = flatbuf.root(data)
    subgraphs = m.tables(2)
    if len(subgraphs) != 1:
        raise ValueError(f"expected one subgraph, found {len(subgraphs)}")
    codes = []
    for oc in m.tables(1):
        # builtin_code (slot 3) supersedes deprecated_builtin_code (slot 0)
        codes.append(max(oc.scalar(3, "i", 0), oc.scalar(0, "b", 0)))
    buffers = []
    for b in m.tables(4):
        loc = b.vector_bytes(0)
        buffers.append(loc if loc is not None and loc[1] > 0 else None)
    sg = subgraphs[0]
    tensors = []
    for t in sg.tables(0):
        q = t.table(4)
        scale, zp, qdim = [], [], 0
        if q is not None:
            scale = q.vector(2, "f")
            zp = q.vector(3, "q")
            qdim = q.scalar(6, "i", 0)
        tensors.append(TensorInfo(tuple(t.vector(0, "i")), t.scalar(1, "b", 0), t.scalar(2, "I", 0),
                                  t.string(3) or "", scale, zp, qdim))
    ops = []
    for o in sg.tables(3):
        otype = o.scalar(3, "B", 0)
        idx = o.scalar(0, "I", 0)
        if idx >= len(codes):
            raise ValueError("operator code index out of range")
        ops.append(OpInfo(codes[idx], o.vector(1, "i"), o.vector(2, "i"), otype,
                          _options(o, otype)))
    return TfliteModel(data, tensors, ops, sg.vector(1, "i"), sg.vector(2, "i"), buffers)


# --------------------------------------------------------- int8 lowering
def quantize_multiplier(real: float) -> tuple[int, int]:
    """TFLite QuantizeMultiplier (the same function as netspec's)."""
    return netspec.quantize_multiplier(real)


def activation_range(act: int, scale: float, zp: int) -> tuple[int, int]:
    """TFLite CalculateActivationRangeQuantized for int8 outputs."""
    qmin, qmax = -128, 127

    def q(v):
        r = v / scale  # TfLiteRound: half away from zero
        return zp + int(math.floor(abs(r) + 0.5)) * (1 if r >= 0 else -1)

    if act == ACT_NONE:
        return qmin, qmax
    if act == ACT_RELU:
        return max(qmin, q(0.0)), qmax
    if act == ACT_RELU6:
        return max(qmin, q(0.0)), min(qmax, q(6.0))
    if act == ACT_RELU_N1_TO_1:
        return max(qmin, q(-1.0)), min(qmax, q(1.0))
    raise ValueError(f"unsupported fused activation {act}")


def _hwc(shape) -> tuple[int, int, int]:
    s = list(shape)
    if len(s) == 4:
        return int(s[1]), int(s[2]), int(s[3])
    if len(s) == 2:
        return 1, 1, int(s[1])
    if len(s) == 3:
        return 1, int(s[1]), int(s[2])
    raise ValueError(f"unsupported tensor shape {shape}")


def _quant(ti: TensorInfo, what: str) -> tuple[float, int]:
    if ti.type != T_INT8 or not ti.scale:
        raise ValueError(f"{what}: expected a quantized int8 tensor")
    return float(np.float32(ti.scale[0])), int(ti.zero_point[0]) if ti.zero_point else 0


def _pads(padding, h, w, kh, kw, sh, sw):
    if padding == PAD_VALID:
        return (0, 0, 0, 0)
    if padding == PAD_SAME:
        return tuple(netspec.same_padding(h, w, kh, kw, sh, sw))
    raise ValueError(f"unsupported padding {padding}")


def to_network(model: TfliteModel, name: str = "tflite") -> netspec.Network:
    """Lowers an int8 model (operators in a chain) to a netspec.Network."""
    if len(model.inputs) != 1 or len(model.outputs) != 1:
        raise ValueError("expected one input and one output tensor")
    x = model.inputs[0]
    in_ti = model.tensors[x]
    s_in0, zp_in0 = _quant(in_ti, "model input")
    layers = []
    cur = x
    for i, op in enumerate(model.operators):
        if not op.inputs or op.inputs[0] != cur:
            raise ValueError(f"operator {i} ({op.name}) does not read the previous output: "
                             "only chains are supported")
        t_in = model.tensors[op.inputs[0]]
        t_out = model.tensors[op.outputs[0]]
        s_in, zp_in = _quant(t_in, f"{op.name} input")
        s_out, zp_out = _quant(t_out, f"{op.name} output")
        ishape, oshape = _hwc(t_in.shape), _hwc(t_out.shape)
        o = op.options
        tag = f"op{i}_{op.name.lower()}"
        if op.code in (OP_CONV_2D, OP_DEPTHWISE_CONV_2D):
            dw = op.code == OP_DEPTHWISE_CONV_2D
            if o.get("dilation_w", 1) != 1 or o.get("dilation_h", 1) != 1:
                raise ValueError(f"{op.name}: dilation is not supported")
            if dw and o.get("depth_multiplier", 1) != 1:
                raise ValueError("DEPTHWISE_CONV_2D: depth_multiplier must be 1")
            w_ti = model.tensors[op.inputs[1]]
            w = model.constant(op.inputs[1])
            if w is None or w_ti.type != T_INT8:
                raise ValueError(f"{op.name}: constant int8 weights expected")
            if any(z != 0 for z in w_ti.zero_point):
                raise ValueError(f"{op.name}: weights must be symmetric (zero point 0)")
            co = oshape[2]
            kh, kw = (w.shape[1], w.shape[2])
            filt = (w.reshape(kh, kw, co) if dw else w).astype(np.int8).copy()
            sh, sw = o["stride_h"], o["stride_w"]
            pad = _pads(o["padding"], ishape[0], ishape[1], kh, kw, sh, sw)
            kind = capi.OP_DEPTHWISE_CONV2D if dw else capi.OP_CONV2D
        elif op.code == OP_FULLY_CONNECTED:
            if o.get("weights_format", 0) != 0:
                raise ValueError("FULLY_CONNECTED: only the default weights format")
            w_ti = model.tensors[op.inputs[1]]
            w = model.constant(op.inputs[1])
            if w is None or w_ti.type != T_INT8 or any(z != 0 for z in w_ti.zero_point):
                raise ValueError("FULLY_CONNECTED: constant symmetric int8 weights expected")
            co = int(w.shape[0])
            if int(w.shape[1]) != int(np.prod(ishape)):
                raise ValueError("FULLY_CONNECTED: weights do not match the input size")
            filt = w.astype(np.int8).copy()
            kind, kh, kw, sh, sw, pad = capi.OP_FULLY_CONNECTED, 1, 1, 1, 1, (0, 0, 0, 0)
            oshape = (1, 1, co)
        elif op.code in (OP_MAX_POOL_2D, OP_AVERAGE_POOL_2D):
            if abs(s_in - s_out) > 1e-6 * s_in or zp_in != zp_out:
                raise ValueError(f"{op.name}: input and output quantization must match")
            kh, kw, sh, sw = o["filter_h"], o["filter_w"], o["stride_h"], o["stride_w"]
            pad = _pads(o["padding"], ishape[0], ishape[1], kh, kw, sh, sw)
            kind = capi.OP_MAX_POOL2D if op.code == OP_MAX_POOL_2D else capi.OP_AVERAGE_POOL2D
            amin, amax = activation_range(o.get("activation", 0), s_out, zp_out)
            l = netspec.Layer(kind, ishape, oshape, (kh, kw), (sh, sw), pad, False, zp_in=zp_in,
                              zp_out=zp_out, s_in=s_in, s_out=s_out, act_min=amin, act_max=amax,
                              name=tag)
            layers.append(l)
            cur = op.outputs[0]
            continue
        elif op.code == OP_RESHAPE:
            l = netspec.Layer(capi.OP_RESHAPE, ishape, oshape, zp_in=zp_in, zp_out=zp_out,
                              s_in=s_in, s_out=s_out, name=tag)
            layers.append(l)
            cur = op.outputs[0]
            continue
        else:
            raise ValueError(f"unsupported operator: {op.name}")

        # weighted op: bias, per-channel multipliers, activation range
        w_scale = np.array([float(np.float32(v)) for v in w_ti.scale], dtype=np.float64)
        if w_scale.size == 1:
            w_scale = np.full(co, w_scale[0])
        if w_scale.size != co:
            raise ValueError(f"{op.name}: {w_scale.size} weight scales for {co} channels")
        bias = np.zeros(co, np.int32)
        if len(op.inputs) > 2 and op.inputs[2] >= 0:
            b = model.constant(op.inputs[2])
            if b is None or model.tensors[op.inputs[2]].type != T_INT32:
                raise ValueError(f"{op.name}: int32 bias expected")
            bias = b.astype(np.int32).reshape(co).copy()
        mult = np.zeros(co, np.int32)
        shift = np.zeros(co, np.int32)
        for c in range(co):
            mult[c], shift[c] = quantize_multiplier(s_in * w_scale[c] / s_out)
        amin, amax = activation_range(o.get("activation", 0), s_out, zp_out)
        expect_h = (ishape[0] + pad[0] + pad[1] - kh) // sh + 1
        expect_w = (ishape[1] + pad[2] + pad[3] - kw) // sw + 1
        if kind != capi.OP_FULLY_CONNECTED and (expect_h, expect_w) != oshape[:2]:
            raise ValueError(f"{op.name}: output shape {oshape} does not match the padding")
        l = netspec.Layer(kind, ishape, oshape, (kh, kw), (sh, sw), pad,
                          o.get("activation", 0) != ACT_NONE, filt, bias, w_scale, zp_in, zp_out,
                          s_in, s_out, mult, shift, amin, amax, name=tag)
        layers.append(l)
        cur = op.outputs[0]
    if cur != model.outputs[0]:
        raise ValueError("the last operator does not write the model output")
    return netspec.Network(name, layers, _hwc(in_ti.shape), s_in0, zp_in0,
                           input_kind="uniform_int8")


# ------------------------------------------------------------------ writing
def _tensor(shape, ttype, buf, name, scale=None, zp=None, qdim=0) -> flatbuf.Obj:
    t = flatbuf.Obj()
    t.ref(0, flatbuf.Vec("i", [int(v) for v in shape]))
    t.scalar(1, "b", ttype)
    t.scalar(2, "I", buf)
    t.ref(3, flatbuf.Str(name))
    if scale is not None:
        q = flatbuf.Obj()
        q.ref(2, flatbuf.Vec("f", [float(np.float32(v)) for v in scale]))
        q.ref(3, flatbuf.Vec("q", [int(v) for v in zp]))
        q.scalar(6, "i", qdim)
        t.ref(4, q)
    return t


def write_network(net: netspec.Network, description: str = "psp-ml-b200 int8 model") -> bytes:
    """Serialises an int8 network as a .tflite model (one subgraph, batch 1
    shapes; weights per-channel symmetric, biases int32)."""
    tensors, buffers, ops, codes = [], [flatbuf.Obj()], [], []

    def code_index(c):
        if c not in codes:
            codes.append(c)
        return codes.index(c)

    def const(arr: np.ndarray) -> int:
        b = flatbuf.Obj().ref(0, flatbuf.Vec("B", np.ascontiguousarray(arr).tobytes(), align=16))
        buffers.append(b)
        return len(buffers) - 1

    def act_tensor(shape_hwc, scale, zp, name, rank4=True):
        shape = [1, *shape_hwc] if rank4 else [1, int(np.prod(shape_hwc))]
        tensors.append(_tensor(shape, T_INT8, 0, name, [scale], [zp]))
        return len(tensors) - 1

    cur = act_tensor(net.in_shape, net.in_scale, net.in_zp, "input")
    for l in net.layers:
        opt = flatbuf.Obj()
        if l.kind in (capi.OP_CONV2D, capi.OP_DEPTHWISE_CONV2D, capi.OP_FULLY_CONNECTED):
            co = l.out_shape[2]
            ws = [float(v) for v in l.w_scale]
            if l.kind == capi.OP_CONV2D:
                wshape, qdim, code = l.filter.shape, 0, OP_CONV_2D
            elif l.kind == capi.OP_DEPTHWISE_CONV2D:
                wshape, qdim, code = (1, *l.filter.shape), 3, OP_DEPTHWISE_CONV_2D
            else:
                wshape, qdim, code = l.filter.shape, 0, OP_FULLY_CONNECTED
            tensors.append(_tensor(wshape, T_INT8, const(l.filter), f"{l.name}/w", ws, [0] * co,
                                   qdim))
            wt = len(tensors) - 1
            bscale = [float(np.float32(l.s_in)) * float(np.float32(v)) for v in ws]
            tensors.append(_tensor([co], T_INT32, const(l.bias.astype(np.int32)), f"{l.name}/b",
                                   bscale, [0] * co, 0))
            bt = len(tensors) - 1
            fc = l.kind == capi.OP_FULLY_CONNECTED
            out = act_tensor(l.out_shape if not fc else (co,), l.s_out, l.zp_out, l.name,
                             rank4=not fc)
            act = ACT_RELU if l.relu else ACT_NONE
            if fc:
                opt.scalar(0, "b", act)
                otype = OPT_FULLY_CONNECTED
            else:
                padding = _padding_kind(l)
                opt.scalar(0, "b", padding).scalar(1, "i", l.stride[1]).scalar(2, "i", l.stride[0])
                if l.kind == capi.OP_CONV2D:
                    opt.scalar(3, "b", act)
                    otype = OPT_CONV2D
                else:
                    opt.scalar(3, "i", 1).scalar(4, "b", act)
                    otype = OPT_DEPTHWISE
            inputs = [cur, wt, bt]
        elif l.kind in (capi.OP_MAX_POOL2D, capi.OP_AVERAGE_POOL2D):
            code = OP_MAX_POOL_2D if l.kind == capi.OP_MAX_POOL2D else OP_AVERAGE_POOL_2D
            out = act_tensor(l.out_shape, l.s_out, l.zp_out, l.name)
            opt.scalar(0, "b", _padding_kind(l)).scalar(1, "i", l.stride[1])
            opt.scalar(2, "i", l.stride[0]).scalar(3, "i", l.kernel[1]).scalar(4, "i", l.kernel[0])
            otype = OPT_POOL2D
            inputs = [cur]
        elif l.kind == capi.OP_RESHAPE:
            code = OP_RESHAPE
            out = act_tensor(l.out_shape, l.s_out, l.zp_out, l.name)
            opt.ref(0, flatbuf.Vec("i", [1, *l.out_shape]))
            otype = OPT_RESHAPE
            inputs = [cur]
        else:
            raise ValueError(f"layer kind {l.kind} cannot be written")
        o = flatbuf.Obj()
        o.scalar(0, "I", code_index(code))
        o.ref(1, flatbuf.Vec("i", inputs))
        o.ref(2, flatbuf.Vec("i", [out]))
        o.scalar(3, "B", otype)
        o.ref(4, opt)
        ops.append(o)
        cur = out
    sg = flatbuf.Obj()
    sg.ref(0, flatbuf.Vec("table", tensors))
    sg.ref(1, flatbuf.Vec("i", [0]))
    sg.ref(2, flatbuf.Vec("i", [cur]))
    sg.ref(3, flatbuf.Vec("table", ops))
    sg.ref(4, flatbuf.Str("main"))
    opcodes = []
    for c in codes:
        oc = flatbuf.Obj()
        oc.scalar(0, "b", min(c, 127)).scalar(2, "i", 1).scalar(3, "i", c)
        opcodes.append(oc)
    m = flatbuf.Obj()
    m.scalar(0, "I", 3)
    m.ref(1, flatbuf.Vec("table", opcodes))
    m.ref(2, flatbuf.Vec("table", [sg]))
    m.ref(3, flatbuf.Str(description))
    m.ref(4, flatbuf.Vec("table", buffers))
    return flatbuf.build(m, identifier=b"TFL3")


def _padding_kind(l: netspec.Layer) -> int:
    """VALID for a layer without padding (its output size is the VALID one),
    SAME when the padding is what SAME gives."""
    if tuple(l.pad) == (0, 0, 0, 0):
        return PAD_VALID
    same = netspec.same_padding(l.in_shape[0], l.in_shape[1], l.kernel[0], l.kernel[1],
                                l.stride[0], l.stride[1])
    if tuple(same) == tuple(l.pad):
        return PAD_SAME
    raise ValueError(f"{l.name}: padding {l.pad} is neither SAME nor VALID")


# ------------------------------------------------------------- f32 lowering
@dataclass
class F32Op:
    kind: str                # "conv2d", "max_pool2d", "reshape", "fully_connected"
    in_shape: tuple
    out_shape: tuple
    params: dict = field(default_factory=dict)
    weights: np.ndarray | None = None
    bias: np.ndarray | None = None


def to_f32_plan(model: TfliteModel) -> list[F32Op]:
    """Lowers a float32 model to the ops of the reference's f32 kernels
    (lowering.rs:156-306): CONV_2D (+ReLU), MAX_POOL_2D 2x2 stride 2,
    RESHAPE, FULLY_CONNECTED (+ReLU)."""
    plan = []
    for op in model.operators:
        t_in = model.tensors[op.inputs[0]]
        t_out = model.tensors[op.outputs[0]]
        if t_in.type != T_FLOAT32:
            raise ValueError(f"{op.name}: float32 tensors expected")
        o = op.options
        if op.code == OP_CONV_2D:
            w = model.constant(op.inputs[1])
            kh, kw = int(w.shape[1]), int(w.shape[2])
            pad = _pads(o["padding"], t_in.shape[1], t_in.shape[2], kh, kw, o["stride_h"],
                        o["stride_w"])
            b = model.constant(op.inputs[2]) if len(op.inputs) > 2 and op.inputs[2] >= 0 else None
            act = o.get("activation", 0)
            if act not in (ACT_NONE, ACT_RELU):
                raise ValueError("CONV_2D: only ReLU or no activation on the f32 path")
            plan.append(F32Op("conv2d", tuple(t_in.shape), tuple(t_out.shape),
                              dict(stride=(o["stride_h"], o["stride_w"]), pad=pad,
                                   relu=act == ACT_RELU),
                              np.ascontiguousarray(w, np.float32),
                              None if b is None else np.ascontiguousarray(b, np.float32)))
        elif op.code == OP_MAX_POOL_2D:
            if (o["filter_h"], o["filter_w"], o["stride_h"], o["stride_w"]) != (2, 2, 2, 2):
                raise ValueError("MAX_POOL_2D: only 2x2 stride 2 (as the reference)")
            plan.append(F32Op("max_pool2d", tuple(t_in.shape), tuple(t_out.shape)))
        elif op.code == OP_RESHAPE:
            plan.append(F32Op("reshape", tuple(t_in.shape), tuple(t_out.shape)))
        elif op.code == OP_FULLY_CONNECTED:
            w = model.constant(op.inputs[1])
            b = model.constant(op.inputs[2]) if len(op.inputs) > 2 and op.inputs[2] >= 0 else None
            act = o.get("activation", 0)
            if act not in (ACT_NONE, ACT_RELU):
                raise ValueError("FULLY_CONNECTED: only ReLU or no activation on the f32 path")
            plan.append(F32Op("fully_connected", tuple(t_in.shape), tuple(t_out.shape),
                              dict(relu=act == ACT_RELU), np.ascontiguousarray(w, np.float32),
                              None if b is None else np.ascontiguousarray(b, np.float32)))
        else:
            raise ValueError(f"unsupported operator: {op.name}")
    return plan
