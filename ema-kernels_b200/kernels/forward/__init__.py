"""EMA forward (ema_fwd_triton, chunk_cumsum_triton)."""
