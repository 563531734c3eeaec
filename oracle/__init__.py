"""CPU oracle (test infrastructure only): restatement of the reference's fp32
blockscale GEMM, client/aiter/hsa/gfx942/driver.py:18-20.  Never imported by
the product package."""
