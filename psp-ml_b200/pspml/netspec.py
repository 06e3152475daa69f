"""Synthetic int8 networks for the psp-ml inference path.

The reference compiles a TFLite model into an op chain whose constants sit at
offsets in one weight blob (cargo-psp-ml/src/parse/tflite/lowering.rs:26-124,
TensorKind::Constant in cargo-psp-ml/src/ir/graph.rs:22-31).  This module
builds the same thing for the five benchmark workloads, with seeded synthetic
weights, and emits it in the C-ABI form (pspml_op_desc array + blob):

  config 0  small CNN 28x28x1: conv3x3(8)+ReLU, maxpool, conv3x3(16)+ReLU,
            maxpool, reshape, FC 784->10
  config 1  single FC [B,K] x [K,K]^T sweep, fixed multipliers / shifts
  config 2  64x64x3 CNN: 4 stages of [conv3x3+ReLU, conv3x3+ReLU, maxpool]
            over 32/64/128/256 channels, global avg pool, FC 256->100
  config 3  depthwise-separable CNN on [96,512,1]: stem conv3x3/s2 to 32 ch
            +ReLU, 8 blocks of [DW3x3+ReLU, PW1x1], global avg pool,
            FC 512->3337
  config 4  config 3's network at global batch 262144

Quantisation follows TFLite: activations int8 with a per-tensor zero point,
weights symmetric int8 per output channel (scales log-uniform in
[1e-3, 1e-1]), int32 bias at scale s_in*s_w.  Output scales come from a
deterministic float64 calibration pass over a few seeded samples (99.9th
percentile of the layer's real output).  The per-channel multiplier/shift
pairs use TFLite's QuantizeMultiplier.
"""
from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass, field

import numpy as np

from . import capi

# Synthetic-input stand-ins for the reference's datasets (MNIST images are
# not shipped with the reference; BirdNET spectrograms are not available).
# float32-representable (a .tflite file stores float32 scales)
CFG_IN_SCALE = {k: float(np.float32(v)) for k, v in {0: 1.0 / 255.0, 2: 1.0 / 255.0, 3: 0.1}.items()}
CFG_IN_ZP = {0: -128, 2: -128, 3: 0}

CFG3_WIDTHS = (64, 64, 128, 128, 256, 256, 512, 512)
CFG3_DW_STRIDES = (1, 1, 2, 1, 2, 1, 2, 1)


def rng_for(tag: str) -> np.random.Generator:
    """Independent deterministic stream per tensor name."""
    seed = int.from_bytes(hashlib.sha256(tag.encode()).digest()[:8], "little")
    return np.random.default_rng(seed)


def quantize_multiplier(real: float) -> tuple[int, int]:
    """TFLite QuantizeMultiplier: real = M * 2**(shift - 31), M in [2**30, 2**31)."""
    if real == 0.0:
        return 0, 0
    q, e = math.frexp(real)
    q_fixed = int(math.floor(abs(q) * (1 << 31) + 0.5)) * (1 if q >= 0 else -1)
    if q_fixed == (1 << 31):
        q_fixed //= 2
        e += 1
    if e < -31:
        e, q_fixed = 0, 0
    if e > 30:
        e, q_fixed = 30, (1 << 31) - 1
    return q_fixed, e


def same_padding(in_h: int, in_w: int, k_h: int, k_w: int, s_h: int, s_w: int):
    """(top, bottom, left, right) as cargo-psp-ml/src/parse/tflite/lowering.rs:341-364."""
    oh = (in_h + s_h - 1) // s_h
    ow = (in_w + s_w - 1) // s_w
    th = max((oh - 1) * s_h + k_h - in_h, 0)
    tw = max((ow - 1) * s_w + k_w - in_w, 0)
    return th // 2, th - th // 2, tw // 2, tw - tw // 2


@dataclass
class Layer:
    kind: int
    in_shape: tuple[int, int, int]
    out_shape: tuple[int, int, int]
    kernel: tuple[int, int] = (1, 1)
    stride: tuple[int, int] = (1, 1)
    pad: tuple[int, int, int, int] = (0, 0, 0, 0)  # top, bottom, left, right
    relu: bool = False
    filter: np.ndarray | None = None
    bias: np.ndarray | None = None
    w_scale: np.ndarray | None = None
    zp_in: int = 0
    zp_out: int = 0
    s_in: float = 1.0
    s_out: float = 1.0
    mult: np.ndarray | None = None
    shift: np.ndarray | None = None
    act_min: int = -128
    act_max: int = 127
    name: str = ""

    @property
    def macs_per_sample(self) -> int:
        ho, wo, co = self.out_shape
        if self.kind == capi.OP_CONV2D:
            return ho * wo * co * self.kernel[0] * self.kernel[1] * self.in_shape[2]
        if self.kind == capi.OP_DEPTHWISE_CONV2D:
            return ho * wo * co * self.kernel[0] * self.kernel[1]
        if self.kind == capi.OP_FULLY_CONNECTED:
            return co * int(np.prod(self.in_shape))
        return 0

    @property
    def weight_bytes(self) -> int:
        n = 0
        for a in (self.filter, self.bias, self.mult, self.shift):
            if a is not None:
                n += a.nbytes
        return n


@dataclass
class Network:
    name: str
    layers: list[Layer]
    in_shape: tuple[int, int, int]
    in_scale: float
    in_zp: int
    input_kind: str = "uniform_pixels"
    meta: dict = field(default_factory=dict)

    @property
    def in_elems(self) -> int:
        return int(np.prod(self.in_shape))

    @property
    def out_elems(self) -> int:
        return int(np.prod(self.layers[-1].out_shape))

    def macs_per_sample(self) -> int:
        return sum(l.macs_per_sample for l in self.layers)

    def descs_and_blob(self) -> tuple[np.ndarray, np.ndarray]:
        """The C-ABI form: pspml_op_desc array and the weight blob."""
        descs = np.zeros(len(self.layers), dtype=capi.OP_DESC_DTYPE)
        parts: list[bytes] = []
        off = 0

        def put(a: np.ndarray | None) -> int:
            nonlocal off
            if a is None:
                return -1
            pad = (-off) % 256
            if pad:
                parts.append(b"\0" * pad)
                off += pad
            here = off
            b = np.ascontiguousarray(a).tobytes()
            parts.append(b)
            off += len(b)
            return here

        for i, l in enumerate(self.layers):
            d = descs[i]
            d["kind"] = l.kind
            d["in_h"], d["in_w"], d["in_c"] = l.in_shape
            d["out_h"], d["out_w"], d["out_c"] = l.out_shape
            d["kernel_h"], d["kernel_w"] = l.kernel
            d["stride_h"], d["stride_w"] = l.stride
            d["pad_top"], d["pad_bottom"], d["pad_left"], d["pad_right"] = l.pad
            d["zp_in"], d["zp_out"] = l.zp_in, l.zp_out
            d["act_min"], d["act_max"] = l.act_min, l.act_max
            d["filter_off"] = put(l.filter)
            d["bias_off"] = put(l.bias)
            d["mult_off"] = put(l.mult)
            d["shift_off"] = put(l.shift)
        blob = np.frombuffer(b"".join(parts), dtype=np.uint8).copy()
        return descs, blob

    def make_input(self, n: int, tag: str = "input") -> np.ndarray:
        """Seeded synthetic int8 input batch [n, H, W, C]."""
        r = rng_for(f"{self.name}/{tag}/{n}")
        shape = (n,) + tuple(self.in_shape)
        if self.input_kind == "gaussian_spectrogram":
            v = np.rint(r.normal(-40.0, 25.0, size=shape))
            return np.clip(v, -128, 127).astype(np.int8)
        if self.input_kind == "uniform_int8":
            return r.integers(-128, 128, size=shape, dtype=np.int16).astype(np.int8)
        pixels = r.integers(0, 256, size=shape, dtype=np.int16)
        return (pixels - 128).astype(np.int8)


# ------------------------------------------------------------ float64 model
# Used only to pick output scales (calibration), like the TFLite converter's
# representative-dataset pass.  Padding is real zero.

def _conv_f(x, w, b, stride, pad, depthwise=False):
    n, h, wd, c = x.shape
    pt, pb, pl, pr = pad
    sh, sw = stride
    if depthwise:
        kh, kw, _ = w.shape
    else:
        _, kh, kw, _ = w.shape
    xp = np.pad(x, ((0, 0), (pt, pb), (pl, pr), (0, 0)))
    ho = (h + pt + pb - kh) // sh + 1
    wo = (wd + pl + pr - kw) // sw + 1
    co = c if depthwise else w.shape[0]
    y = np.zeros((n, ho, wo, co), dtype=np.float64)
    for i in range(kh):
        for j in range(kw):
            xs = xp[:, i:i + (ho - 1) * sh + 1:sh, j:j + (wo - 1) * sw + 1:sw, :]
            if depthwise:
                y += xs * w[i, j, :]
            else:
                y += (xs.reshape(-1, c) @ w[:, i, j, :].T).reshape(n, ho, wo, co)
    return y + b


def _pool_f(x, kernel, stride, mode):
    n, h, w, c = x.shape
    kh, kw = kernel
    sh, sw = stride
    ho = (h - kh) // sh + 1
    wo = (w - kw) // sw + 1
    acc = None
    for i in range(kh):
        for j in range(kw):
            xs = x[:, i:i + (ho - 1) * sh + 1:sh, j:j + (wo - 1) * sw + 1:sw, :]
            if acc is None:
                acc = xs.copy()
            elif mode == "max":
                acc = np.maximum(acc, xs)
            else:
                acc = acc + xs
    return acc if mode == "max" else acc / (kh * kw)


def _f32(v: float) -> float:
    return float(np.float32(v))


class _Builder:
    """Appends layers, calibrating each weighted layer's output scale."""

    def __init__(self, name, in_shape, in_scale, in_zp, calib_x_real):
        self.name = name
        self.layers: list[Layer] = []
        self.shape = tuple(in_shape)
        # Scales are kept float32-representable: a .tflite file stores them
        # as float32 and TFLite derives the multipliers from those values.
        self.scale = _f32(in_scale)
        self.zp = in_zp
        self.x = calib_x_real  # float64 activations of the calibration batch

    def _weights(self, tag, shape, co):
        r = rng_for(f"{self.name}/{tag}/w")
        q = r.integers(-127, 128, size=shape, dtype=np.int16).astype(np.int8)
        rs = rng_for(f"{self.name}/{tag}/ws")
        ws = np.exp(rs.uniform(math.log(1e-3), math.log(1e-1), size=co))
        ws = ws.astype(np.float32).astype(np.float64)
        rb = rng_for(f"{self.name}/{tag}/b")
        bq = rb.integers(-4096, 4097, size=co, dtype=np.int64).astype(np.int32)
        return q, ws, bq

    def _finish(self, l: Layer, y_real: np.ndarray):
        if l.relu:
            y_real = np.maximum(y_real, 0.0)
            pos = y_real[y_real > 0]
            pct = float(np.percentile(pos, 99.9)) if pos.size else 1.0
            l.s_out = _f32(max(pct, 1e-6) / 255.0)
            l.zp_out = -128
        else:
            pct = float(np.percentile(np.abs(y_real), 99.9)) if y_real.size else 1.0
            l.s_out = _f32(max(pct, 1e-6) / 127.0)
            l.zp_out = 0
        l.act_min = max(-128, l.zp_out) if l.relu else -128
        l.act_max = 127
        m = np.zeros(l.out_shape[2], dtype=np.int32)
        s = np.zeros(l.out_shape[2], dtype=np.int32)
        for c in range(l.out_shape[2]):
            m[c], s[c] = quantize_multiplier(l.s_in * float(l.w_scale[c]) / l.s_out)
        l.mult, l.shift = m, s
        self.layers.append(l)
        self.x = y_real
        self.shape, self.scale, self.zp = l.out_shape, l.s_out, l.zp_out

    def conv(self, tag, co, k=3, stride=1, padding="same", relu=True):
        h, w, c = self.shape
        if padding == "same":
            pad = same_padding(h, w, k, k, stride, stride)
        else:
            pad = (0, 0, 0, 0)
        ho = (h + pad[0] + pad[1] - k) // stride + 1
        wo = (w + pad[2] + pad[3] - k) // stride + 1
        q, ws, bq = self._weights(tag, (co, k, k, c), co)
        l = Layer(capi.OP_CONV2D, (h, w, c), (ho, wo, co), (k, k), (stride, stride), pad, relu,
                  q, bq, ws, self.zp, 0, self.scale, name=tag)
        wr = q.astype(np.float64) * ws[:, None, None, None]
        br = bq.astype(np.float64) * self.scale * ws
        self._finish(l, _conv_f(self.x, wr, br, (stride, stride), pad))

    def dwconv(self, tag, k=3, stride=1, relu=True):
        h, w, c = self.shape
        pad = same_padding(h, w, k, k, stride, stride)
        ho = (h + pad[0] + pad[1] - k) // stride + 1
        wo = (w + pad[2] + pad[3] - k) // stride + 1
        q, ws, bq = self._weights(tag, (k, k, c), c)
        l = Layer(capi.OP_DEPTHWISE_CONV2D, (h, w, c), (ho, wo, c), (k, k), (stride, stride), pad,
                  relu, q, bq, ws, self.zp, 0, self.scale, name=tag)
        wr = q.astype(np.float64) * ws[None, None, :]
        br = bq.astype(np.float64) * self.scale * ws
        self._finish(l, _conv_f(self.x, wr, br, (stride, stride), pad, depthwise=True))

    def fc(self, tag, n_out, relu=False):
        h, w, c = self.shape
        k = h * w * c
        q, ws, bq = self._weights(tag, (n_out, k), n_out)
        l = Layer(capi.OP_FULLY_CONNECTED, (h, w, c), (1, 1, n_out), relu=relu, filter=q,
                  bias=bq, w_scale=ws, zp_in=self.zp, s_in=self.scale, name=tag)
        wr = q.astype(np.float64) * ws[:, None]
        br = bq.astype(np.float64) * self.scale * ws
        y = self.x.reshape(self.x.shape[0], -1) @ wr.T + br
        self._finish(l, y.reshape(-1, 1, 1, n_out))

    def _passthrough(self, l: Layer, y):
        l.zp_in = l.zp_out = self.zp
        l.s_in = l.s_out = self.scale
        l.act_min, l.act_max = -128, 127
        self.layers.append(l)
        self.x = y
        self.shape = l.out_shape

    def maxpool(self, tag, k=2, s=2):
        h, w, c = self.shape
        ho, wo = (h - k) // s + 1, (w - k) // s + 1
        l = Layer(capi.OP_MAX_POOL2D, (h, w, c), (ho, wo, c), (k, k), (s, s), name=tag)
        self._passthrough(l, _pool_f(self.x, (k, k), (s, s), "max"))

    def global_avgpool(self, tag):
        h, w, c = self.shape
        l = Layer(capi.OP_AVERAGE_POOL2D, (h, w, c), (1, 1, c), (h, w), (h, w), name=tag)
        self._passthrough(l, _pool_f(self.x, (h, w), (h, w), "avg"))

    def reshape(self, tag, shape):
        l = Layer(capi.OP_RESHAPE, self.shape, tuple(shape), name=tag)
        self._passthrough(l, self.x.reshape((self.x.shape[0],) + tuple(shape)))


def _calib_input(net_stub: Network, n: int) -> np.ndarray:
    q = net_stub.make_input(n, tag="calibration").astype(np.float64)
    return (q - net_stub.in_zp) * net_stub.in_scale


def build_config0(calib_samples: int = 16) -> Network:
    stub = Network("cfg0_mnist_s8", [], (28, 28, 1), CFG_IN_SCALE[0], CFG_IN_ZP[0])
    b = _Builder(stub.name, stub.in_shape, stub.in_scale, stub.in_zp,
                 _calib_input(stub, calib_samples))
    b.conv("conv1", 8)
    b.maxpool("pool1")
    b.conv("conv2", 16)
    b.maxpool("pool2")
    b.reshape("reshape", (1, 1, 784))
    b.fc("fc", 10)
    stub.layers = b.layers
    return stub


def build_config2(calib_samples: int = 4) -> Network:
    stub = Network("cfg2_cnn64_s8", [], (64, 64, 3), CFG_IN_SCALE[2], CFG_IN_ZP[2])
    b = _Builder(stub.name, stub.in_shape, stub.in_scale, stub.in_zp,
                 _calib_input(stub, calib_samples))
    for si, c in enumerate((32, 64, 128, 256)):
        b.conv(f"s{si}a", c)
        b.conv(f"s{si}b", c)
        b.maxpool(f"s{si}pool")
    b.global_avgpool("gap")
    b.fc("fc", 100)
    stub.layers = b.layers
    return stub


def build_config3(calib_samples: int = 4) -> Network:
    stub = Network("cfg3_birdnet_dwsep_s8", [], (96, 512, 1), CFG_IN_SCALE[3], CFG_IN_ZP[3],
                   input_kind="gaussian_spectrogram")
    b = _Builder(stub.name, stub.in_shape, stub.in_scale, stub.in_zp,
                 _calib_input(stub, calib_samples))
    b.conv("stem", 32, k=3, stride=2)
    for i, (wd, s) in enumerate(zip(CFG3_WIDTHS, CFG3_DW_STRIDES)):
        b.dwconv(f"b{i}_dw", stride=s)
        b.conv(f"b{i}_pw", wd, k=1, relu=False)
    b.global_avgpool("gap")
    b.fc("fc", 3337)
    stub.layers = b.layers
    return stub


def build_fc_sweep(batch: int, k: int) -> Network:
    """Config 1: one FC [B,K] x [K,K]^T.  Activations U[-128,127] with zp -3;
    weights U[-127,127]; bias int32 in +-2**12; multipliers uniform in
    [2**30, 2**31); right shifts uniform in 5..12; output zp 5 with ReLU."""
    name = f"cfg1_fc_b{batch}_k{k}"
    r = rng_for(name)
    w = r.integers(-127, 128, size=(k, k), dtype=np.int16).astype(np.int8)
    bias = r.integers(-4096, 4097, size=k, dtype=np.int64).astype(np.int32)
    mult = r.integers(1 << 30, 1 << 31, size=k, dtype=np.int64).astype(np.int32)
    shift = -r.integers(5, 13, size=k, dtype=np.int64).astype(np.int32)
    l = Layer(capi.OP_FULLY_CONNECTED, (1, 1, k), (1, 1, k), relu=True, filter=w, bias=bias,
              zp_in=-3, zp_out=5, mult=mult, shift=shift, act_min=5, act_max=127, name="fc")
    return Network(name, [l], (1, 1, k), 1.0, -3, input_kind="uniform_int8",
                   meta={"batch": batch, "k": k})


BUILDERS = {0: build_config0, 2: build_config2, 3: build_config3}
