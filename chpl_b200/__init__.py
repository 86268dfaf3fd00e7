"""chpl_b200 -- a B200-native (sm_100a) HPL engine with the drop-in surface of
Koyingtw/CHPL: the Ozaki-II emulated trailing update (GEMMul8 interface), the
FP64 panel/pivoting path and the chpl_single / chpl_p2 solvers.

All compute runs in the in-tree CUDA library libchpl.so (C ABI: include/chpl.h);
importing a submodule that needs it raises if the library is missing.
"""
from ._lib import ChplError, load  # noqa: F401

__all__ = ["ChplError", "load", "oz2", "hpl"]
__version__ = "0.1"
