"""B200-native (sm_100a) implementation of MuSc's scoring hot path.

* ``musc_b200.ops``      -- torch-facing wrappers of the C ABI (include/musc_b200.h)
* ``musc_b200.pipeline`` -- device-resident pool scoring on 1..G GPUs
* ``musc_b200.backend``  -- the ``b200`` inference backend for MuSc's seam
* ``musc_b200.synthetic``-- seeded prototype-mixture inputs
"""
from ._lib import LIB_PATH, LibraryMissing  # noqa: F401

__all__ = ['LIB_PATH', 'LibraryMissing']
