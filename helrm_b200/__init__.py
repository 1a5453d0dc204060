"""B200-native CKKS backend for HE-LRM's embedding PCMM.

The operator surface lives in :class:`helrm_b200.library.B200Library`; the
kernels in ``csrc/`` are compiled to ``libhelrm_b200.so`` by
:mod:`helrm_b200.build` and reached through the C ABI declared in
``include/helrm_b200.h``.
"""
from .library import B200Library  # noqa: F401
from .params import CKKSConfig  # noqa: F401
