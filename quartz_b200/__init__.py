"""quartz_b200: B200-native (sm_100a) fused int8 weight-only matmul path."""
