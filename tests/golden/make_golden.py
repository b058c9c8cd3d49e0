"""Generates the golden fixtures in this directory from the reference itself.

Run once, in a checkout that has the reference package available (the path of the
kernelpilot source tree is the first, required, argument):

    python tests/golden/make_golden.py /path/to/kernelpilot [op ...]

For every op, dtype and shape below it calls the reference's own input generator
(``spec.make_inputs(shape, dtype, cpu, seed=0)``, kernelpilot/specs.py:69-72) and its
float64 reference (``spec.reference``), and stores inputs and outputs in
``<op>.npz``. The causal attention fixtures use PyTorch's float64
``scaled_dot_product_attention(..., is_causal=True)``, the reference's own baseline
call with the causal flag, since the reference has no causal op.

bf16 tensors are stored as raw uint16 bit patterns. Keys: ``<dtype>|<shape>|in<i>``
and ``<dtype>|<shape>|out``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent

SHAPES = {
    "vector_add": [(1,), (7,), (1000,), (1024,), (65537,)],
    "reduce_sum": [(1,), (7,), (1000,), (1024,), (65537,)],
    "softmax": [(1, 1), (1, 7), (3, 1000), (17, 1024), (5, 4097), (2, 129)],
    "matmul": [(1, 1, 1), (7, 13, 5), (64, 64, 64), (127, 129, 65), (33, 100, 77)],
    "layernorm": [(1, 1), (1, 7), (3, 1000), (17, 1024), (5, 4097), (2, 129)],
    "attention": [(1, 1, 1, 16), (1, 2, 7, 32), (1, 2, 64, 64), (1, 2, 100, 64),
                  (1, 3, 50, 48), (1, 1, 40, 128)],
}
SHAPES["attention_causal"] = SHAPES["attention"]
DTYPES = [torch.float32, torch.float16, torch.bfloat16]


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def main(ref_root: str, ops: list[str]) -> None:
    sys.path.insert(0, ref_root)
    from kernelpilot.specs import get_spec  # the reference's own contract

    cpu = torch.device("cpu")
    for op, shapes in SHAPES.items():
        if ops and op not in ops:
            continue
        spec = get_spec("attention" if op == "attention_causal" else op)
        blob: dict[str, np.ndarray] = {}
        for dtype in DTYPES:
            dname = str(dtype).replace("torch.", "")
            for shape in shapes:
                inputs = spec.make_inputs(shape, dtype, cpu, 0)
                if op == "attention_causal":
                    q, k, v = (t.double() for t in inputs)
                    out = F.scaled_dot_product_attention(q, k, v, is_causal=True)
                else:
                    out = spec.reference(*inputs)
                key = f"{dname}|{','.join(map(str, shape))}"
                for i, t in enumerate(inputs):
                    blob[f"{key}|in{i}"] = to_np(t)
                blob[f"{key}|out"] = out.double().numpy()
        np.savez_compressed(HERE / f"{op}.npz", **blob)
        print(op, len(blob) // 2, "arrays")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/kernelpilot [op ...]")
    main(sys.argv[1], sys.argv[2:])
