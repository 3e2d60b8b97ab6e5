"""jax4j_b200 -- B200 (sm_100a) execution backend for jax4j.

The public API mirrors the reference's Java API (NDArray, JAX, Lax, Nn,
Numpy, Random, PyTree, Device, Shape, DType) on device-resident arrays; all
computation runs in libjax4j_cuda.so (include/jax4j_cuda.h).
"""
from .core import (ConcreteNDArray, Device, DType, IllegalArgumentException, IllegalStateException,
                   NDArray, PRNGKey, Primitive, Shape, UnsupportedOperationException)
from .tracing import Equation, Jaxpr, Tracer, TracedNDArray, Var
from .pytree import PyTree, PyTrees
from .api import Fft, JAX, Lax, Linalg, Nn, Numpy, Random, SingularityCheck, Svd
from .pmap import CollectiveError, LocalShard, PmapContext
from ._lib import J4CError, J4CTimeout

__all__ = ["ConcreteNDArray", "Device", "DType", "NDArray", "PRNGKey", "Primitive", "Shape",
           "IllegalArgumentException", "IllegalStateException", "UnsupportedOperationException",
           "Equation", "Jaxpr", "Tracer", "TracedNDArray", "Var", "PyTree", "PyTrees", "JAX", "Lax",
           "Nn", "Numpy", "Random", "Fft", "Linalg", "SingularityCheck", "Svd", "CollectiveError", "LocalShard", "PmapContext", "J4CError",
           "J4CTimeout"]
