"""CPU oracle: a restatement of lesiondiffusion-mlx's hot-path arithmetic.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and
the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import
this package, and only as the checker or the timed CPU baseline.  The
product path (``lesiondiffusion_mlx_b200``) never imports it and has no CPU
fallback.

The reference (MLX 0.32 + Metal, Darwin arm64 only) cannot run on Linux, so
this package restates its algorithms in PyTorch-CPU / NumPy following the
reference source op for op (each function cites the file:line it follows,
paths relative to ``src/lesiondiffusion_mlx/`` of lesiondiffusion-mlx 0.3.0).
It is pinned against the reference's own golden vectors (Torch-CPU recordings
of the pinned upstream model, committed under ``tests/golden/``) by
``tests/test_oracle_golden.py``.  Arithmetic that lives in the un-vendored
medmlx-core 0.3.0 (group normalization) is restated from its call sites and
pinned only through those recordings at their tolerances; its bitwise
reduction order is unpinned.
"""
