"""exactsample_b200: exactsample's batch-invariant sampling and speculative
verification on B200 (sm_100a).

The public surface is the reference package's CUDA API
(python/exactsample/__init__.py, cuda.py, types.py): ``plan``, ``verify``,
``CudaPlan``, ``CudaRequestParams``, ``CudaRngKey``, ``CudaOutput``,
``load_library`` and the ``Status`` / ``PathUsed`` / ``RequestParams`` /
``RngKey`` / ``VerifyOutput`` types. The FP64 NumPy oracle of the reference
is not part of this package.
"""
from .types import PathUsed, RequestParams, RngKey, Status, VerifyOutput

__version__ = "0.1.0"


def plan(*args, **kwargs):
    from .cuda import plan as implementation
    return implementation(*args, **kwargs)


def verify(*args, **kwargs):
    from .cuda import verify as implementation
    return implementation(*args, **kwargs)


__all__ = ["PathUsed", "RequestParams", "RngKey", "Status", "VerifyOutput", "plan", "verify"]
