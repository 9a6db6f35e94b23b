"""Test infrastructure: the CPU oracle for qrb200.

``qr_oracle``  -- numpy float32 restatement of the reference pipeline
                  (reflection_no_reflectors.py:55-196), pinned by ``tests/golden``.
``checker``    -- fp64 residual / orthogonality / tau gates (common/oracle.py:156-195).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (CPU baseline and the
``--impl reference`` arm) may import this package, and only as a checker or as the
timed CPU baseline -- never as part of the shipped CUDA path.
"""
