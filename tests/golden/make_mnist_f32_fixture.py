"""Writes tests/golden/mnist_cnn_f32.npz: the float32 weights and biases of
the reference's MNIST model (examples/mnist-bench/mnist_cnn.tflite), as the
reference's own parser locates them (generated.rs:317-336), read with this
repository's TFLite reader.  The GPU f32 tests run the model from this
fixture, since the reference tree is not available where they run.

    python tests/golden/make_mnist_f32_fixture.py [path/to/mnist_cnn.tflite]

The default path is the reference checkout named by PSPML_REFERENCE_ROOT
(or a `reference` directory beside this repository).
"""
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "psp-ml_b200"))

from pspml import tflite  # noqa: E402

OUT = HERE / "mnist_cnn_f32.npz"


def reference_model_path() -> Path:
    base = Path(os.environ.get("PSPML_REFERENCE_ROOT", ROOT.parent / "reference"))
    return base / "examples" / "mnist-bench" / "mnist_cnn.tflite"


def main(argv):
    src = Path(argv[1]) if len(argv) > 1 else reference_model_path()
    plan = tflite.to_f32_plan(tflite.load(src))
    kinds = [p.kind for p in plan]
    assert kinds == ["conv2d", "max_pool2d", "conv2d", "max_pool2d", "reshape",
                     "fully_connected", "fully_connected"], kinds
    conv1, conv2, fc1, fc2 = plan[0], plan[2], plan[5], plan[6]
    arrays = {}
    for name, p in (("conv1", conv1), ("conv2", conv2), ("fc1", fc1), ("fc2", fc2)):
        arrays[f"{name}_w"] = p.weights
        arrays[f"{name}_b"] = p.bias
        arrays[f"{name}_relu"] = np.array(p.params["relu"])
    arrays["conv_pad"] = np.array([conv1.params["pad"], conv2.params["pad"]], np.int64)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} from {src}")


if __name__ == "__main__":
    main(sys.argv)
