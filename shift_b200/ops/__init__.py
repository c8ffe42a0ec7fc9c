"""sm_100a kernels and their fp32 reference statements."""
from . import functional, gemm, reference  # noqa: F401
from ._ext import available, check_status, ext  # noqa: F401
