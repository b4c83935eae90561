"""EMA backward and autograd (compute_dpx, ema_combined)."""
