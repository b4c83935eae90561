"""CPU oracle for the EMA / Mamba-2 SSD chunked scan (TEST INFRASTRUCTURE ONLY).

Nothing in the product package imports this directory.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) may import it, and only as the checker or as the
timed CPU baseline -- never as the thing that is measured or shipped.

Modules
-------
``ema_oracle``      float64 numpy restatement of the reference's EMA forward
                    (``ema_fwd_triton``), backward (``compute_dpx``), the
                    ``ema_combined`` autograd pair, ``chunk_cumsum_triton`` and
                    the dt-parameterised EMA used by the benchmark configs.
``ssd_oracle``      float64 numpy Mamba-2 SSD recurrence and its adjoint (the
                    reference calls a third-party package for this; the oracle
                    is written from the recurrence itself).
``ema_torch_path``  restatement of the reference's PyTorch CPU path
                    (``ema_torch_ref`` + autograd) used as the timed CPU
                    baseline.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own kernels
under the Triton CPU interpreter (fp32) and stores their outputs as fixtures;
``tests/test_oracle_golden.py`` checks this oracle against every fixture.
The SSD oracle has no reference implementation to pin against ("parity
unpinned" for the SSD rows); it is cross-checked against torch autograd of
its own forward recurrence instead.
"""
