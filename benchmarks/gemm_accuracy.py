"""Accuracy of the tcgen05 GEMM modes against an fp64 reference.

Prints, for each K, the max relative error (max |C - C_ref| / max |C_ref|) of
abacus tf32 (1 pass), abacus fp32 (3xTF32) and cuBLAS SGEMM (TF32 off, the
reference framework's numerics).

    python benchmarks/gemm_accuracy.py
"""
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from abacus_b200.ops import gemm, precision  # noqa: E402


def main():
    torch.backends.cuda.matmul.allow_tf32 = False
    for k in (64, 256, 768, 2048, 8192, 65536):
        torch.manual_seed(k)
        m, n = 512, 768
        a = torch.randn(m, k, device="cuda")
        b = torch.randn(k, n, device="cuda")
        ref = a.double() @ b.double()
        scale = ref.abs().max().item()
        row = {"k": k}
        for mode in ("tf32", "fp32"):
            precision.set_precision(mode)
            row[f"abacus_{mode}"] = (gemm.matmul(a, b).double() - ref).abs().max().item() / scale
        precision.set_precision("fp32")
        row["cublas_sgemm"] = ((a @ b).double() - ref).abs().max().item() / scale
        print(json.dumps({key: (f"{v:.2e}" if isinstance(v, float) else v) for key, v in row.items()}), flush=True)


if __name__ == "__main__":
    main()
