"""Generates the golden fixtures in tests/golden/ from the reference itself.

Runs the reference's own CPU path (Bee::Tensor public ops, compiled from the
reference sources by oracle/Makefile into oracle/_ref/libbee_ref.so) on small
seeded inputs and stores inputs and outputs as .npz files.  The fixtures pin
the oracle restatement (tests/test_oracle_pins.py) and the CUDA kernels
(tests/test_gpu_*.py) without needing the reference at test time.

    make -C oracle ref && python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle.oracle import Reference, bf16_round  # noqa: E402


def main():
    ref = Reference()
    rng = np.random.default_rng(20261201)
    out = {}

    # fp32 GEMM: odd (tail) shapes and a blocking-sized one (GemmTests.cpp:93-128 style)
    for (m, k, n) in [(17, 13, 11), (33, 65, 47), (128, 96, 160)]:
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        c, _ = ref.matmul_f32(a, b)
        out[f"matmul_f32_{m}x{k}x{n}"] = dict(a=a, b=b, c=c)

    # elementwise add / mul, odd length
    a = rng.standard_normal((7, 1031)).astype(np.float32)
    b = rng.standard_normal((7, 1031)).astype(np.float32)
    out["add_f32"] = dict(a=a, b=b, c=ref.binary_f32(0, a, b)[0])
    out["mul_f32"] = dict(a=a, b=b, c=ref.binary_f32(2, a, b)[0])

    # row sum / max (short rows -> warp path, long rows -> CTA path)
    for (r, c) in [(33, 257), (5, 4099)]:
        x = rng.standard_normal((r, c)).astype(np.float32)
        out[f"row_sum_f32_{r}x{c}"] = dict(x=x, y=ref.reduce_rows_f32(0, x)[0])
        out[f"row_max_f32_{r}x{c}"] = dict(x=x, y=ref.reduce_rows_f32(2, x)[0])

    # int32 full sum, the odd sizes of Tests/CUDA/ReduceTests.cu:88-169
    for n in [1, 31, 32, 256, 257, 4096, (1 << 16) + 3]:
        x = rng.integers(-1000, 1001, n).astype(np.int32)
        out[f"sum_i32_{n}"] = dict(x=x, y=np.array([ref.reduce_global_i32(0, x)[0]], np.int32))

    # softmax rows
    for (r, c) in [(16, 300), (4, 8192)]:
        x = rng.standard_normal((r, c)).astype(np.float32)
        out[f"softmax_f32_{r}x{c}"] = dict(x=x, y=ref.softmax_f32(x)[0])

    # RMSNorm on bf16-rounded inputs (the bf16 config's math in fp32)
    x = bf16_round(rng.standard_normal((8, 4096)).astype(np.float32))
    w = bf16_round((1.0 + 0.02 * rng.standard_normal(4096)).astype(np.float32))
    out["rms_norm_bf16in_8x4096"] = dict(x=x, w=w, y=ref.rms_norm_f32(x, w, 1e-6)[0])

    # RoPE on [batch 2, seq 4, heads 4, head_dim 128], bf16-rounded inputs
    x = bf16_round(rng.standard_normal((8, 4 * 128)).astype(np.float32))
    out["rope_bf16in_2x4x4x128"] = dict(x=x, y=ref.rope_f32(x, 4, 4, 128, 10000.0, 0)[0])

    # attention chain on [heads 2, seq 64, hd 32], bf16-rounded inputs
    q, k, v = (bf16_round(rng.standard_normal((2, 64, 32)).astype(np.float32)) for _ in range(3))
    scale = float(1.0 / np.sqrt(32.0))
    out["attention_bf16in_2x64x32"] = dict(q=q, k=k, v=v, o=ref.attention_f32(q, k, v, scale)[0])

    for name, arrays in out.items():
        np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print(f"wrote {len(out)} fixtures to {HERE}")


if __name__ == "__main__":
    main()
