"""sparsefold_b200: B200-native (sm_100a) kernels for the AF3 trunk hot path of SparseFold.

The package is a drop-in backend for SparseFold's plugin API
(``sparsefold_b200.backend.register``) and also ships standalone modules with
the reference parameter layout (``sparsefold_b200.modules``).  All arithmetic
runs in ``libsparsefold_b200.so`` (C ABI, ``include/sparsefold_b200.h``).
"""

__version__ = "0.1.0"
