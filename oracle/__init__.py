"""CPU oracle for the tensorshrink QuantLinear hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the `tensorshrink_b200` package imports
this directory; only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline
legs of `bench.py` use it, and only as the checker (or the timed CPU
baseline), never as the thing measured or shipped.

`goap.py` restates, in numpy, the reference algorithms the CUDA kernels must
match: GOAP quantize (top-k outliers, group affine, NF / Lloyd-Max codebooks,
bit packing, double quantization), dequantize, the outlier-delta precompute of
`QuantLinear`, and the fp32 dequant-matmul that defines the GEMM tolerance.
Parity is pinned by `tests/test_oracle_golden.py` against fixtures generated
by running the reference itself (`tests/golden/make_golden.py`).
"""
