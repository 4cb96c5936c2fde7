"""CPU oracle for basal's quantised-linear hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the CPU arithmetic of the reference (rkinas/basal 2.8.1):

  oracle.fp8        e4m3 / e2m1 codecs (torch's float8_e4m3fn cast; basal/nvfp4.py:19-46 e2m1 table and cuts)
  oracle.blockquant FP8-block and INT8-block formats (basal/blockquant.py:54-60, :118-135; fp8block.py:30-31;
                    int8block.py:43-44)
  oracle.nvfp4      NVFP4 codes, 128x4 scale swizzle, weight/activation quantisers, CPU linear
                    (basal/nvfp4.py:36-112, :197-213)
  oracle.readout    the option-code readout (basal/readout.py:39-104)

It is the checker, never the product: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
(`--impl reference` and the `cpu_baseline` field) may import it. The product package basal_b200 never imports it
and fails loudly when its CUDA library is missing.

Pinning: tests/golden/make_golden.py imports the reference itself (read-only, in the build container) and writes
the fixtures under tests/golden/; tests/test_oracle_golden.py checks every function here against them bit for bit
(codes, scales) or to fp32 rounding (GEMM and readout outputs).
"""
