"""TFLite front end (pspml.tflite, pspml.flatbuf) on the CPU.

* The reader against the reference's own model file and its parser's
  output: the constant-tensor locations the reference's generated code
  records for mnist_cnn.tflite (tests/golden/ref_mnist_tflite_offsets.py),
  and the op list and shapes its lowering produces (lowering.rs:19-124).
  These tests read the reference tree and are skipped where it is absent.
* int8 round trips: a config network written as .tflite and read back
  lowers to the same op descriptors and weight blob, and the oracle gives
  the same logits.
* Rejections the reference's lowering also makes (unsupported operators),
  and those of the int8 path (graphs that are not chains, asymmetric
  weights)."""
import math
import os
from pathlib import Path

import numpy as np
import pytest

from golden.ref_mnist_tflite_offsets import MNIST_CONSTANTS, MNIST_FILE_BYTES
from pspml import capi, flatbuf, netspec, tflite

# The reference checkout: PSPML_REFERENCE_ROOT, else a `reference` directory
# beside this repository.
REF_ROOT = Path(os.environ.get("PSPML_REFERENCE_ROOT",
                               Path(__file__).resolve().parents[2] / "reference"))
REF_MNIST = REF_ROOT / "examples" / "mnist-bench" / "mnist_cnn.tflite"
needs_ref = pytest.mark.skipif(not REF_MNIST.exists(), reason="reference tree not present")
FIXTURE = Path(__file__).resolve().parent / "golden" / "mnist_cnn_f32.npz"


@needs_ref
def test_mnist_fixture_holds_the_reference_weights():
    """tests/golden/mnist_cnn_f32.npz (used by the GPU f32 test) holds exactly
    the reference model's constants at the reference parser's offsets."""
    m = tflite.load(REF_MNIST)
    raw = np.frombuffer(m.data, np.float32)
    fx = np.load(FIXTURE)
    # tensor indices of conv1/conv2/fc1/fc2 weights and biases in the file
    plan = tflite.to_f32_plan(m)
    for name, p in (("conv1", plan[0]), ("conv2", plan[2]), ("fc1", plan[5]), ("fc2", plan[6])):
        np.testing.assert_array_equal(fx[f"{name}_w"], p.weights)
        np.testing.assert_array_equal(fx[f"{name}_b"], p.bias)
    foff, flen = MNIST_CONSTANTS[8]
    np.testing.assert_array_equal(fx["conv1_w"].reshape(-1), raw[foff:foff + flen])


@needs_ref
def test_reference_mnist_constant_locations_match_reference_parser():
    m = tflite.load(REF_MNIST)
    assert len(m.data) == MNIST_FILE_BYTES
    for t, (foff, flen) in MNIST_CONSTANTS.items():
        off, n = m.buffers[m.tensors[t].buffer]
        assert (off // 4, n // 4) == (foff, flen), f"tensor {t}"
        assert off % 4 == 0


@needs_ref
def test_reference_mnist_ops_and_f32_plan():
    m = tflite.load(REF_MNIST)
    assert [o.name for o in m.operators] == ["CONV_2D", "MAX_POOL_2D", "CONV_2D", "MAX_POOL_2D",
                                             "RESHAPE", "FULLY_CONNECTED", "FULLY_CONNECTED"]
    plan = tflite.to_f32_plan(m)
    assert [(p.kind, p.out_shape) for p in plan] == [
        ("conv2d", (1, 28, 28, 8)), ("max_pool2d", (1, 14, 14, 8)),
        ("conv2d", (1, 14, 14, 16)), ("max_pool2d", (1, 7, 7, 16)),
        ("reshape", (1, 784)), ("fully_connected", (1, 64)), ("fully_connected", (1, 10))]
    # SAME 5x5 stride 1 -> 2 on every side (lowering.rs:366-420)
    assert plan[0].params == dict(stride=(1, 1), pad=(2, 2, 2, 2), relu=True)
    assert plan[5].params["relu"] and not plan[6].params["relu"]
    assert plan[0].weights.shape == (8, 5, 5, 1) and plan[5].weights.shape == (64, 784)
    # the weights are the file's bytes at the reference's offsets
    raw = np.frombuffer(m.data, np.float32)
    foff, flen = MNIST_CONSTANTS[8]
    np.testing.assert_array_equal(plan[0].weights.reshape(-1), raw[foff:foff + flen])


@needs_ref
def test_reference_mnist_runs_through_the_f32_oracle(oracle_mod):
    """The imported plan drives the f32 oracle (the reference's kernel
    semantics) to 10 finite logits; a float64 restatement agrees."""
    m = tflite.load(REF_MNIST)
    plan = tflite.to_f32_plan(m)
    x = np.random.default_rng(3).random((1, 28, 28, 1), dtype=np.float32)
    h = x.reshape(-1)
    ref = x.astype(np.float64)
    for p in plan:
        if p.kind == "conv2d":
            h = oracle_mod.f32_conv2d(h, p.in_shape, p.weights.reshape(-1), p.weights.shape,
                                      p.bias, p.params["stride"], p.params["pad"], p.out_shape,
                                      relu=p.params["relu"])
            ref = _conv_f64(ref, p)
        elif p.kind == "max_pool2d":
            h = oracle_mod.f32_max_pool2d(h, p.in_shape, (2, 2), (2, 2), p.out_shape)
            n, hh, ww, c = ref.shape
            ref = ref.reshape(n, hh // 2, 2, ww // 2, 2, c).max(axis=(2, 4))
        elif p.kind == "reshape":
            ref = ref.reshape(1, -1)
        else:
            h = oracle_mod.f32_fully_connected(h, p.in_shape[-1], p.weights.reshape(-1), p.bias,
                                               p.out_shape[-1], relu=p.params["relu"])
            ref = ref.reshape(1, -1) @ p.weights.astype(np.float64).T + p.bias
            if p.params["relu"]:
                ref = np.maximum(ref, 0)
    assert h.shape == (10,) and np.all(np.isfinite(h))
    np.testing.assert_allclose(h, ref.reshape(-1), rtol=1e-4, atol=1e-4)


def _conv_f64(x, p):
    n, hh, ww, ci = x.shape
    w = p.weights.astype(np.float64)
    co, kh, kw, _ = w.shape
    pt, pb, pl, pr = p.params["pad"]
    xp = np.pad(x, ((0, 0), (pt, pb), (pl, pr), (0, 0)))
    ho, wo = p.out_shape[1], p.out_shape[2]
    out = np.zeros((n, ho, wo, co))
    for ky in range(kh):
        for kx in range(kw):
            out += np.einsum("nhwc,oc->nhwo", xp[:, ky:ky + ho, kx:kx + wo, :], w[:, ky, kx, :])
    out += p.bias
    return np.maximum(out, 0) if p.params["relu"] else out


@pytest.mark.parametrize("cfg", [0, 2, 3])
def test_int8_network_round_trip(oracle_mod, cfg):
    net = netspec.BUILDERS[cfg]()
    data = tflite.write_network(net)
    assert flatbuf.file_identifier(data) == b"TFL3"
    back = tflite.to_network(tflite.load(data))
    d0, b0 = net.descs_and_blob()
    d1, b1 = back.descs_and_blob()
    assert d0.tobytes() == d1.tobytes()
    assert b0.tobytes() == b1.tobytes()
    if cfg == 0:
        x = net.make_input(4)
        np.testing.assert_array_equal(oracle_mod.net_forward_s8(d0, b0, x),
                                      oracle_mod.net_forward_s8(d1, b1, x))


def test_depthwise_and_average_pool_options_survive():
    net = netspec.BUILDERS[3]()
    m = tflite.load(tflite.write_network(net))
    names = [o.name for o in m.operators]
    assert names.count("DEPTHWISE_CONV_2D") == 8 and names.count("AVERAGE_POOL_2D") == 1
    dw = next(o for o in m.operators if o.name == "DEPTHWISE_CONV_2D")
    assert dw.options["depth_multiplier"] == 1 and dw.options["activation"] == tflite.ACT_RELU
    # per-channel weight scales on the channel dimension (3 of [1,KH,KW,C])
    w = m.tensors[dw.inputs[1]]
    assert w.quantized_dimension == 3 and len(w.scale) == w.shape[3]


def test_activation_ranges():
    assert tflite.activation_range(tflite.ACT_NONE, 0.1, 5) == (-128, 127)
    assert tflite.activation_range(tflite.ACT_RELU, 0.1, -128) == (-128, 127)
    assert tflite.activation_range(tflite.ACT_RELU, 0.1, 5) == (5, 127)
    assert tflite.activation_range(tflite.ACT_RELU6, 0.05, -128) == (-128, -8)
    assert tflite.activation_range(tflite.ACT_RELU_N1_TO_1, 0.01, 0) == (-100, 100)
    # half away from zero (TfLiteRound), not to even
    assert tflite.activation_range(tflite.ACT_RELU6, 0.8, 0) == (0, 8)


def _tiny_model(ops, tensors_extra=()):
    """A hand-built model: input [1,4,4,16] int8 -> ops (opcode list)."""
    def tensor(shape, name):
        q = flatbuf.Obj().ref(2, flatbuf.Vec("f", [0.5])).ref(3, flatbuf.Vec("q", [0]))
        return (flatbuf.Obj().ref(0, flatbuf.Vec("i", shape)).scalar(1, "b", tflite.T_INT8)
                .scalar(2, "I", 0).ref(3, flatbuf.Str(name)).ref(4, q))
    tensors = [tensor([1, 4, 4, 16], "in"), tensor([1, 4, 4, 16], "a"),
               tensor([1, 4, 4, 16], "b")]
    opcodes = [flatbuf.Obj().scalar(3, "i", c) for c in sorted(set(c for c, _, _ in ops))]
    code_ids = sorted(set(c for c, _, _ in ops))
    operators = [flatbuf.Obj().scalar(0, "I", code_ids.index(c)).ref(1, flatbuf.Vec("i", i))
                 .ref(2, flatbuf.Vec("i", o)) for c, i, o in ops]
    sg = (flatbuf.Obj().ref(0, flatbuf.Vec("table", tensors)).ref(1, flatbuf.Vec("i", [0]))
          .ref(2, flatbuf.Vec("i", [ops[-1][2][0]])).ref(3, flatbuf.Vec("table", operators)))
    m = (flatbuf.Obj().scalar(0, "I", 3).ref(1, flatbuf.Vec("table", opcodes))
         .ref(2, flatbuf.Vec("table", [sg])).ref(4, flatbuf.Vec("table", [flatbuf.Obj()])))
    return flatbuf.build(m, b"TFL3")


def test_unsupported_operator_rejected():
    data = _tiny_model([(tflite.OP_SOFTMAX, [0], [1])])
    with pytest.raises(ValueError, match="unsupported operator: SOFTMAX"):
        tflite.to_network(tflite.load(data))


def test_non_chain_rejected():
    # the second op reads the model input, not the first op's output
    data = _tiny_model([(tflite.OP_RESHAPE, [0], [1]), (tflite.OP_RESHAPE, [0], [2])])
    with pytest.raises(ValueError, match="only chains"):
        tflite.to_network(tflite.load(data))


def test_flatbuffer_round_trip_scalars_vectors_tables():
    inner = flatbuf.Obj().scalar(0, "q", -(1 << 40)).ref(1, flatbuf.Str("héllo"))
    root = (flatbuf.Obj().scalar(0, "B", 7).scalar(2, "i", -5).scalar(3, "d", math.pi)
            .ref(4, flatbuf.Vec("q", [1, -2, 1 << 50]))
            .ref(5, flatbuf.Vec("B", bytes(range(40)), align=16))
            .ref(6, flatbuf.Vec("table", [inner, flatbuf.Obj()]))
            .ref(7, inner))
    buf = flatbuf.build(root, b"ABCD")
    t = flatbuf.root(buf)
    assert flatbuf.file_identifier(buf) == b"ABCD"
    assert t.scalar(0, "B") == 7 and t.scalar(1, "i", 99) == 99 and t.scalar(2, "i") == -5
    assert t.scalar(3, "d") == math.pi
    assert t.vector(4, "q") == [1, -2, 1 << 50]
    off, n = t.vector_bytes(5)
    assert n == 40 and off % 16 == 0 and buf[off:off + n] == bytes(range(40))
    subs = t.tables(6)
    assert subs[0].scalar(0, "q") == -(1 << 40) and subs[0].string(1) == "héllo"
    assert not subs[1].has(0) and t.table(7).string(1) == "héllo"
