"""mote_b200 -- B200 (sm_100a) CUDA data plane for Mote's Q4_0 linear and
per-token layer kernels.

The compute lives in ``libmote_cuda.so`` (C ABI: ``include/mote_cuda.h``);
this package is the host-side mirror of the reference's Rust wrappers:

* :mod:`mote_b200.context` -- ``CudaContext`` / ``CudaStorage`` / ``Tensor``
* :mod:`mote_b200.ops` -- typed operators with the reference's validation
* :mod:`mote_b200.kernel` -- ``KernelKey`` / ``KernelRegistry`` / ``Runtime``
* :mod:`mote_b200.types` -- dtypes, Q4_0 geometry, tensor descriptors
* :mod:`mote_b200.errors` -- the ``HipError`` taxonomy as exceptions

There is no CPU fallback: without the built library every op raises.
"""
from .types import DType, Encoding, Layout, QuantFormat, RopeLayout, TensorDesc, plain, quantized

__all__ = ["DType", "Encoding", "Layout", "QuantFormat", "RopeLayout", "TensorDesc", "plain",
           "quantized"]
