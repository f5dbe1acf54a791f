"""Local operations: einsum lowering, native GEMM, FFT, halo/window/conv, roll."""
