"""Every op can be captured in a CUDA graph (after one eager call has set up the
per-device state) and replays to the eager result bit for bit."""
import pytest
import torch

from kernelpilot_b200 import ext, registry
from kernelpilot_b200.specs import get_spec

pytestmark = pytest.mark.gpu

CASES = [
    ("vector_add", (1_000_003,), torch.bfloat16),
    ("reduce_sum", (1_000_003,), torch.float32),
    ("softmax", (300, 4097), torch.float32),
    ("softmax", (64, 131072), torch.bfloat16),      # thread-block clusters, DSMEM exchange
    ("softmax", (7, 65537), torch.float32),         # clusters on unaligned rows
    ("layernorm", (300, 4097), torch.bfloat16),
    ("matmul", (300, 4097, 192), torch.bfloat16),   # pitch copy of B, then the CTA-pair GEMM (PDL)
    ("matmul", (1024, 1024, 1024), torch.float16),  # CTA pairs (clusters of two)
    ("matmul", (128, 1024, 512), torch.bfloat16),   # M <= 128: the one-CTA kernel
    ("attention", (1, 4, 1000, 128), torch.bfloat16),
    ("attention_causal", (1, 4, 1000, 128), torch.bfloat16),  # main + few-key grids (PDL)
]


@pytest.mark.parametrize("kernel,shape,dtype", CASES,
                         ids=[f"{k}-{s}-{str(d)[6:]}" for k, s, d in CASES])
def test_op_replays_from_a_cuda_graph(kernel, shape, dtype):
    ops = ext.ops()
    variant = registry.BEST_VARIANT[kernel]
    extra = registry.EXTRA_ARGS.get(kernel, ())
    inputs = get_spec(kernel).make_inputs(shape, dtype, torch.device("cuda"), 0)
    op = getattr(ops, kernel)
    eager = op(*inputs, *extra, variant)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        op(*inputs, *extra, variant)  # warm-up on the capture stream
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            captured = op(*inputs, *extra, variant)
    torch.cuda.current_stream().wait_stream(stream)
    captured.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(captured, eager)
