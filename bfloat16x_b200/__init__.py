"""bfloat16x_b200: B200-native BF16X packed-weight decode fused into GEMV/GEMM."""
