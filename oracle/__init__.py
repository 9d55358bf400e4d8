"""CPU oracle for the OrthoSSM Cheby-RKV hot path — TEST INFRASTRUCTURE ONLY.

Nothing in the product (``orthossm_b200``) imports this package.  Only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py`` use it, and only as the checker or as the
timed CPU baseline, never as a code path that produces product results.

Contents
--------
``cheby_ref``      float64 numpy restatement of the reference algorithm
                   (``sdpc_kernel.py`` of Eddym06/OrthoSSM), each function
                   citing the reference lines it follows.
``cheby_ref.c``    the same forward / TTT arithmetic as a multi-threaded C
                   port (OpenMP), built by ``oracle/Makefile`` into
                   ``oracle/libossm_oracle.so`` and loaded by ``cref``.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own Triton
kernels under ``TRITON_INTERPRET=1`` and stores their outputs as fixtures;
``tests/test_oracle_golden.py`` checks this oracle against them.
Modes with no reference implementation (per-token dynamic lambda gate,
W_pred/Adam TTT) are "parity unpinned": the oracle is a restatement of the
published spec, and its gradient is cross-checked against autograd.
"""
