"""B200-native (sm_100a) EMA / Mamba-2 SSD chunked scan.

Drop-in for the reference package ``kernels`` (kartiksrinivas007/ema-kernels):
the same module paths and entry points --

    kernels.forward.ema_ssd_fwd.ema_fwd_triton / chunk_cumsum_triton
    kernels.backward.ema_ssd_combined.compute_dpx / ema_combined / _EmaFunction

-- plus the dt-parameterised EMA used by the benchmark configs
(``kernels.ema_chunk_scan``).  All compute runs in libema_ssd_b200.so
(hand-written CUDA for sm_100a, C ABI in include/ema_ssd_b200.h); importing a
compute module without the built library raises ImportError.
"""
