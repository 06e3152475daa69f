"""Where the reference's TFLite parser places the constant tensors of
examples/mnist-bench/mnist_cnn.tflite: its generated code
(examples/mnist-bench/src/generated.rs:318-335) records, per TFLite tensor
index, the float index of the tensor's data within the model file and its
length in 4-byte elements (the file is included as the weight blob, and
the lowering takes buffer locations by pointer arithmetic,
cargo-psp-ml/src/parse/tflite/lowering.rs:126-155)."""

# tensor index: (float offset into the file, number of 4-byte elements)
MNIST_CONSTANTS = {
    1: (54410, 64),
    2: (54389, 16),
    3: (54376, 10),
    4: (51173, 3200),
    5: (50530, 640),
    6: (351, 50176),
    7: (346, 2),
    8: (143, 200),
    9: (132, 8),
}
MNIST_FILE_BYTES = 220240
