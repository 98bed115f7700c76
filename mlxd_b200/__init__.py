"""mlxd_b200: the per-token decoder step of tlkahn/mlxd on B200 (sm_100a).

The product is the C-ABI library libmlxd_cuda (include/mlxd_cuda.h, sources in
mlxd_b200/csrc). This package only binds it (mlxd_b200.cuda) for the tests and
the benchmark; it has no compute of its own.
"""
from . import cuda  # noqa: F401
