"""CPU oracle for the MuSc scoring hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference's ``original`` backend for the
path the B200 library accelerates:

* ``oracle.lnamd``     -- LNAMD LayerNorm + r x r neighbourhood mean + L2 norm
                          and the super-fast 37->28 adaptive pooling;
* ``oracle.msm``       -- MSM mutual scoring (per-image nearest-patch minima and
                          the interval average);
* ``oracle.reduce``    -- layer/radius means, bilinear up-sampling and the
                          per-image maximum;
* ``oracle.attention`` -- softmax attention of one multi-head block;
* ``oracle.rscin``     -- the RsCIN image-score refinement from class-token
                          similarities;
* ``oracle.torch_cpu`` -- the timed CPU baseline: the reference's LNAMD and MSM
                          with the same torch CPU operations (so its speed is the
                          reference's; pinned bit for bit to the golden outputs).

Every function cites the reference file:line it follows.  Parity is pinned by
``tests/test_oracle_golden.py``, which checks these functions against golden
vectors produced by running the reference itself (``tests/golden``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg (and its ``--impl reference`` arm) may import this package, and only as the checker or the timed CPU
baseline.  The product library never routes through it.
"""
