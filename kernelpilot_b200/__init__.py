"""B200-native (sm_100a) kernels for kernelpilot's torch.ops.kp suite: row softmax,
full sum reduction, GEMM and attention forward, behind the reference's operator
schemas and checked by its float64 correctness contract."""

__version__ = "1.0.0"
