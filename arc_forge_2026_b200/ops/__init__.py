"""CUDA kernels as Python ops (sm_100a), each with a plain-PyTorch oracle used by the tests."""
from ._ext import C, available, check_status

__all__ = ["C", "available", "check_status"]
