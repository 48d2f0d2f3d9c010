"""Host side of the B200 fused RMSNorm+MatMul / MLP backend."""
